// C-ABI entry points (declared in include/w4a16_moe_b200.h): argument checks,
// workspace carving and kernel dispatch.  No allocation, no host sync.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>

#include "../../include/w4a16_moe_b200.h"
#include "launch.cuh"

namespace w4moe {


namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t err, const char* where) {
  return fail(kCudaError, "%s: %s", where, cudaGetErrorString(err));
}

int max_smem_optin() {
  static thread_local int cached_dev = -1, cached = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev != cached_dev) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 0;
    cached_dev = dev;
    cached = v;
  }
  return cached;
}

int sm_count() {
  static thread_local int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    cached_dev = dev;
    cached_sms = sms;
  }
  return cached_sms;
}

// Optional stage events (profiling hook): event i is recorded on the forward's
// stream before align (0), after align (1), after w13 (2) and after w2 (3).
thread_local cudaEvent_t g_stage_events[8];
// Testing hook: route every forward through the general (multi-kernel) path.
thread_local int g_force_general = 0;
thread_local int g_n_stage_events = 0;
// Test hook: 1 = multi-CTA align launches withhold CTA 0's barrier arrival and
// wait ~10 us (the timeout path runs without any fault).
thread_local int g_wait_test = 0;

void mark_stage(int i, cudaStream_t st) {
  if (i >= g_n_stage_events || g_stage_events[i] == nullptr) return;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cap);
  if (cap == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(g_stage_events[i], st, cudaEventRecordExternal);
  else
    cudaEventRecord(g_stage_events[i], st);
}

inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Largest align block size any forward path uses (sizes the shared buffers).
constexpr int64_t kMaxAlignBlock = 128;

struct Workspace {
  int32_t *counts, *offsets, *active, *num_active, *num_post, *tok_valid;
  int32_t *sorted, *expert_ids, *counters, *ready, *sched, *align_bar;
  __nv_bfloat16* inter;
  float* partial;
  int64_t bytes;
};

// Carves the workspace; with base == nullptr only computes the size.
Workspace carve(char* base, int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I) {
  Workspace w{};
  int64_t off = 0;
  auto take = [&](int64_t n) {
    char* p = base ? base + off : nullptr;
    off = align_up(off + n, 256);
    return p;
  };
  const int64_t n_tok = M * topk;
  const int64_t P = align_up(n_tok + E * (kMaxAlignBlock - 1), kMaxAlignBlock);
  // Zero-initialised, self-cleaning state first.
  w.counters = (int32_t*)take(4 * M * (H / 32));
  w.ready = (int32_t*)take(4 * E);
  w.sched = (int32_t*)take(4 * 4);
  w.align_bar = (int32_t*)take(4 * 4);
  w.counts = (int32_t*)take(4 * E);
  w.offsets = (int32_t*)take(4 * (E + 1));
  w.active = (int32_t*)take(4 * E);
  w.num_active = (int32_t*)take(4);
  w.num_post = (int32_t*)take(4);
  w.tok_valid = (int32_t*)take(4 * M);
  w.sorted = (int32_t*)take(4 * P);
  w.expert_ids = (int32_t*)take(4 * P);
  w.inter = (__nv_bfloat16*)take(2 * n_tok * I);
  w.partial = (float*)take(4 * n_tok * H);
  w.bytes = off;
  return w;
}

}  // namespace

// Bytes at the start of a forward workspace that must be zero before a call
// (the self-cleaning counters); everything after them is overwritten by the call.
int64_t workspace_zero_prefix_bytes(int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I) {
  char* const base = reinterpret_cast<char*>(static_cast<uintptr_t>(256));
  Workspace w = carve(base, M, topk, E, H, I);
  return reinterpret_cast<char*>(w.sorted) - base;
}

// Records `msg` as the calling thread's w4a16_last_error() and returns `code`.
int report_error(int code, const char* msg) { return fail(code, "%s", msg); }

}  // namespace w4moe

using namespace w4moe;

extern "C" {

const char* w4a16_last_error(void) { return g_last_error.c_str(); }

int w4a16_version(void) { return 100; }

int w4a16_set_path(int path) {
  g_last_error.clear();
  if (path < 0 || path > 2)
    return fail(kInvalidArgument, "w4a16_set_path: 0 = auto, 1 = general, 2 = tensor-core prefill");
  g_force_general = path;
  return kOk;
}

int w4a16_moe_read_status(const void* workspace, int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I,
                          int32_t* status_out, void* stream) {
  g_last_error.clear();
  if (!workspace || !status_out) return fail(kInvalidArgument, "w4a16_moe_read_status: null pointer");
  Workspace ws = carve((char*)workspace, M, topk, E, H, I);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t err = cudaMemcpyAsync(status_out, ws.sched + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err == cudaSuccess) err = cudaMemsetAsync(ws.sched + 2, 0, sizeof(int32_t), st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_read_status");
  return kOk;
}

int w4a16_set_wait_test(int mode) {
  g_last_error.clear();
  if (mode < 0 || mode > 2) return fail(kInvalidArgument, "w4a16_set_wait_test: mode 0, 1 or 2");
  g_wait_test = mode;
  return kOk;
}

int w4a16_moe_align_read_status(void* scratch, int32_t* status_out, void* stream) {
  g_last_error.clear();
  if (!scratch || !status_out) return fail(kInvalidArgument, "w4a16_moe_align_read_status: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int32_t* bar = (int32_t*)scratch;
  cudaError_t err = cudaMemcpyAsync(status_out, bar + 2, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  // arrivals of a barrier that timed out never reached the CTA count: clear
  // the arrival counter and the error word (the generation word only grows)
  if (err == cudaSuccess && *status_out != 0) err = cudaMemsetAsync(bar, 0, sizeof(int32_t), st);
  if (err == cudaSuccess) err = cudaMemsetAsync(bar + 2, 0, sizeof(int32_t), st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_align_read_status");
  return kOk;
}

int w4a16_set_stage_events(void* const* events, int n_events) {
  g_last_error.clear();
  if (n_events < 0 || n_events > 8 || (n_events > 0 && events == nullptr))
    return fail(kInvalidArgument, "w4a16_set_stage_events: 0 <= n_events <= 8");
  for (int i = 0; i < 8; ++i) g_stage_events[i] = i < n_events ? (cudaEvent_t)events[i] : nullptr;
  g_n_stage_events = n_events;
  return kOk;
}

int64_t w4a16_align_buffer_len(int64_t n_tok, int64_t num_experts, int64_t block_size) {
  if (block_size <= 0 || n_tok < 0 || num_experts <= 0) return -1;
  return align_up(n_tok + num_experts * (block_size - 1), block_size);
}

int64_t w4a16_moe_align_scratch_bytes(int64_t n_tok, int64_t num_experts) {
  if (n_tok < 0 || num_experts <= 0 || num_experts > 1024) return -1;
  if (align_grid_ctas((int)std::min<int64_t>(n_tok, 1LL << 30), (int)num_experts, sm_count()) == 0) return 0;
  return 256 + 4 * (int64_t)align_grid_scratch_ints((int)num_experts, sm_count());
}

int w4a16_moe_align(const void* topk_ids, int ids_is_int64, int64_t M, int64_t topk,
                    int64_t num_experts, int64_t block_size, int32_t* sorted_token_ids,
                    int32_t* expert_ids, int32_t* num_tokens_post_padded, void* stream) {
  return w4a16_moe_align_ex(topk_ids, ids_is_int64, M, topk, num_experts, block_size, sorted_token_ids,
                            expert_ids, num_tokens_post_padded, nullptr, 0, stream);
}

int w4a16_moe_align_ex(const void* topk_ids, int ids_is_int64, int64_t M, int64_t topk,
                       int64_t num_experts, int64_t block_size, int32_t* sorted_token_ids,
                       int32_t* expert_ids, int32_t* num_tokens_post_padded, void* scratch,
                       int64_t scratch_bytes, void* stream) {
  g_last_error.clear();
  if (M < 0 || topk <= 0 || num_experts <= 0 || block_size <= 0)
    return fail(kInvalidArgument, "w4a16_moe_align: bad sizes M=%lld topk=%lld E=%lld bs=%lld",
                (long long)M, (long long)topk, (long long)num_experts, (long long)block_size);
  if (num_experts > 1024)
    return fail(kUnsupported, "w4a16_moe_align: num_experts=%lld > 1024", (long long)num_experts);
  if (M * topk > (1LL << 30))
    return fail(kUnsupported, "w4a16_moe_align: M*topk too large");
  if ((M > 0 && topk_ids == nullptr) || !sorted_token_ids || !expert_ids || !num_tokens_post_padded)
    return fail(kInvalidArgument, "w4a16_moe_align: null pointer");
  AlignParams p{};
  p.map = SlotMap{topk_ids, ids_is_int64 ? 1 : 0, nullptr, 0, (int)num_experts};
  p.n_tok = (int)(M * topk);
  p.topk = (int)topk;
  p.E = (int)num_experts;
  p.bs = (int)block_size;
  p.P = (int)w4a16_align_buffer_len(M * topk, num_experts, block_size);
  p.sorted = sorted_token_ids;
  p.expert_ids = expert_ids;
  p.num_post = num_tokens_post_padded;
  cudaError_t err;
  const int ctas = scratch != nullptr ? align_grid_ctas(p.n_tok, p.E, sm_count()) : 0;
  if (ctas > 0 && scratch_bytes >= w4a16_moe_align_scratch_bytes(p.n_tok, p.E)) {
    p.grid_bar = (int32_t*)scratch;
    if (g_wait_test == 1) {
      p.withhold = 1;
      p.budget = 20000;
    }
    p.scratch = (int32_t*)((char*)scratch + 256);
    err = launch_align_grid(p, ctas, (cudaStream_t)stream);
  } else {
    err = launch_align(p, (cudaStream_t)stream);
  }
  if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_align");
  return kOk;
}

int w4a16_repack(const uint8_t* w_q, const void* scales, int64_t E, int64_t N_out, int64_t K,
                 int64_t group_size, uint8_t* w_rep, void* s_rep, void* stream) {
  g_last_error.clear();
  if (E <= 0 || N_out <= 0 || K <= 0 || !w_q || !scales || !w_rep || !s_rep)
    return fail(kInvalidArgument, "w4a16_repack: bad arguments");
  if (N_out % 16 != 0 || K % 64 != 0)
    return fail(kUnsupported, "w4a16_repack: need N_out %% 16 == 0 and K %% 64 == 0 (N_out=%lld K=%lld)",
                (long long)N_out, (long long)K);
  if (group_size <= 0 || group_size % 32 != 0 || K % group_size != 0)
    return fail(kUnsupported, "w4a16_repack: group_size=%lld must be a multiple of 32 dividing K=%lld",
                (long long)group_size, (long long)K);
  RepackParams p{w_q, (const uint16_t*)scales, (int)E, (int)N_out, (int)K, (int)group_size,
                 (uint32_t*)w_rep, (uint16_t*)s_rep};
  cudaError_t err = launch_repack(p, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "w4a16_repack");
  return kOk;
}

int w4a16_repack_checkpoint(const int32_t* w_packed, const void* scales, int64_t E, int64_t N_out, int64_t K,
                            int64_t group_size, uint8_t* w_rep, void* s_rep, void* stream) {
  g_last_error.clear();
  if (E <= 0 || N_out <= 0 || K <= 0 || !w_packed || !scales || !w_rep || !s_rep)
    return fail(kInvalidArgument, "w4a16_repack_checkpoint: bad arguments");
  if (N_out % 16 != 0 || K % 64 != 0)
    return fail(kUnsupported, "w4a16_repack_checkpoint: need N_out %% 16 == 0 and K %% 64 == 0 (N_out=%lld K=%lld)",
                (long long)N_out, (long long)K);
  if (group_size <= 0 || group_size % 32 != 0 || K % group_size != 0)
    return fail(kUnsupported, "w4a16_repack_checkpoint: group_size=%lld must be a multiple of 32 dividing K=%lld",
                (long long)group_size, (long long)K);
  RepackParams p{nullptr, (const uint16_t*)scales, (int)E, (int)N_out, (int)K, (int)group_size,
                 (uint32_t*)w_rep, (uint16_t*)s_rep, w_packed, 1};
  cudaError_t err = launch_repack(p, (cudaStream_t)stream);
  if (err != cudaSuccess) return cuda_fail(err, "w4a16_repack_checkpoint");
  return kOk;
}

int64_t w4a16_moe_workspace_size(int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I) {
  if (M < 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return -1;
  return carve(nullptr, M, topk, E, H, I).bytes;
}

int w4a16_moe_forward(const void* hidden, int64_t M, int64_t H, int64_t hidden_ld,
                      const void* w13_rep, const void* s13_rep, const void* w2_rep,
                      const void* s2_rep, int64_t E, int64_t I, const float* topk_weights,
                      const void* topk_ids, int ids_is_int64, int64_t topk,
                      const int32_t* expert_map, int64_t global_num_experts, void* out,
                      void* workspace, int64_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (M < 0 || H <= 0 || I <= 0 || E <= 0 || topk <= 0 || hidden_ld < H)
    return fail(kInvalidArgument, "w4a16_moe_forward: bad sizes M=%lld H=%lld I=%lld E=%lld topk=%lld ld=%lld",
                (long long)M, (long long)H, (long long)I, (long long)E, (long long)topk,
                (long long)hidden_ld);
  if (H % 64 != 0 || I % 64 != 0)
    return fail(kUnsupported, "w4a16_moe_forward: need H %% 64 == 0 and I %% 64 == 0 (H=%lld I=%lld)",
                (long long)H, (long long)I);
  if (E > 1024) return fail(kUnsupported, "w4a16_moe_forward: E=%lld > 1024", (long long)E);
  if (M * topk > (1LL << 28)) return fail(kUnsupported, "w4a16_moe_forward: M*topk too large");
  if (expert_map != nullptr && global_num_experts <= 0)
    return fail(kInvalidArgument, "w4a16_moe_forward: expert_map needs global_num_experts > 0");
  if (M == 0) return kOk;
  if (!hidden || !w13_rep || !s13_rep || !w2_rep || !s2_rep || !topk_weights || !topk_ids ||
      !out || !workspace)
    return fail(kInvalidArgument, "w4a16_moe_forward: null pointer");
  if (((uintptr_t)workspace & 255) != 0)
    return fail(kInvalidArgument, "w4a16_moe_forward: workspace must be 256-byte aligned");
  if (((uintptr_t)w13_rep | (uintptr_t)w2_rep) & 15)
    return fail(kInvalidArgument, "w4a16_moe_forward: weights must be 16-byte aligned");
  if (((uintptr_t)s13_rep | (uintptr_t)s2_rep) & 7)
    return fail(kInvalidArgument, "w4a16_moe_forward: scales must be 8-byte aligned");
  if (((uintptr_t)hidden & 3) || (hidden_ld & 1))
    return fail(kInvalidArgument, "w4a16_moe_forward: hidden rows must be 4-byte aligned");
  if ((uintptr_t)out & 15)
    return fail(kInvalidArgument, "w4a16_moe_forward: out must be 16-byte aligned");
  Workspace ws = carve((char*)workspace, M, topk, E, H, I);
  if (workspace_bytes < ws.bytes)
    return fail(kInvalidArgument, "w4a16_moe_forward: workspace %lld bytes < required %lld",
                (long long)workspace_bytes, (long long)ws.bytes);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n_tok = M * topk;
  const SlotMap map{topk_ids, ids_is_int64 ? 1 : 0, expert_map,
                    (int)(expert_map ? global_num_experts : E), (int)E};

  // Small M: one fused persistent kernel (routing + w13 + w2 + top-k sum).
  if (g_force_general == 0 && ((uintptr_t)hidden & 15) == 0 && (hidden_ld & 7) == 0) {
    DecodeParams dp{};
    dp.w13 = (const uint8_t*)w13_rep;
    dp.s13 = (const uint8_t*)s13_rep;
    dp.w2 = (const uint8_t*)w2_rep;
    dp.s2 = (const uint8_t*)s2_rep;
    dp.hidden = (const __nv_bfloat16*)hidden;
    dp.hidden_ld = hidden_ld;
    dp.map = map;
    dp.n_tok = (int)n_tok;
    dp.topk = (int)topk;
    dp.M = (int)M;
    dp.E = (int)E;
    dp.H = (int)H;
    dp.I = (int)I;
    dp.topk_w = topk_weights;
    dp.inter = ws.inter;
    dp.partial = ws.partial;
    dp.out = (__nv_bfloat16*)out;
    dp.counters = ws.counters;
    dp.ready = ws.ready;
    dp.sched = ws.sched;
    dp.zero_rows = expert_map != nullptr;

#ifdef W4A16_DIAGNOSTICS
    if (const char* tr = getenv("W4A16_DECODE_TRACE")) dp.trace = (long long*)strtoull(tr, nullptr, 0);
#endif
    if (decode_plan(dp, sm_count(), max_smem_optin() - 1024)) {
      if (g_wait_test == 2) {  // test hook: readiness withheld, ~10 us waits
        dp.withhold = 1;
        dp.ready_budget = 20000;
      }
      mark_stage(0, st);
      mark_stage(1, st);
      cudaError_t err = launch_decode(dp, st);
      if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_forward/decode");
      mark_stage(2, st);
      mark_stage(3, st);
      return kOk;
    }
  }

  // 1) routing: per-expert counts / offsets / active list (block size 1: the
  //    small-M GEMMs read each expert's exact slot range).
  AlignParams ap{};
  ap.map = map;
  ap.n_tok = (int)n_tok;
  ap.topk = (int)topk;
  ap.E = (int)E;
  ap.bs = 1;
  ap.P = (int)n_tok;
  ap.sorted = ws.sorted;
  ap.expert_ids = ws.expert_ids;
  ap.num_post = ws.num_post;
  ap.counts = ws.counts;
  ap.offsets = ws.offsets;
  ap.active = ws.active;
  ap.num_active = ws.num_active;
  ap.tok_valid = ws.tok_valid;
  ap.zero_rows = (__nv_bfloat16*)out;
  ap.H = (int)H;
  mark_stage(0, st);
  cudaError_t err;
  // chunk totals of the multi-CTA align live in the partial region (free
  // until the GEMMs run)
  const int align_ctas = align_grid_ctas((int)n_tok, (int)E, sm_count());
  if (align_ctas > 0 && (int64_t)align_grid_scratch_ints((int)E, sm_count()) * 4 <= 4 * n_tok * H) {
    ap.scratch = (int32_t*)ws.partial;
    ap.grid_bar = ws.align_bar;
    ap.status = ws.sched + 2;
    err = launch_align_grid(ap, align_ctas, st);
  } else {
    err = launch_align(ap, st);
  }
  if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_forward/align");
  mark_stage(1, st);

  // Large M: tensor-core (tcgen05) grouped GEMMs + fixed-order top-k sum.
  if (g_force_general != 1 && ((uintptr_t)hidden & 15) == 0 && (hidden_ld & 7) == 0 && I % 128 == 0 &&
      H % 128 == 0 && prefill_stages((int)E, max_smem_optin()) > 0) {
    PrefillParams p13{};
    p13.w = (const uint8_t*)w13_rep;
    p13.s = (const uint8_t*)s13_rep;
    p13.n_rowtiles = (int)(2 * I / 16);
    p13.n_chunks = (int)(H / 64);
    p13.x = (const __nv_bfloat16*)hidden;
    p13.x_ld = hidden_ld;
    p13.x_row_div = (int)topk;
    p13.sorted = ws.sorted;
    p13.num_post = ws.num_post;
    p13.n_tok = (int)n_tok;
    // sorted token rows in the upper half of the partial region (the bf16
    // partials of the w2 pass use the lower half)
    p13.xs = (__nv_bfloat16*)ws.partial + n_tok * H;
    p13.offsets = ws.offsets;
    p13.counts = ws.counts;
    p13.active = ws.active;
    p13.num_active = ws.num_active;
    p13.E = (int)E;
    p13.topk = (int)topk;
    p13.I = (int)I;
    p13.H = (int)H;
    p13.inter = ws.inter;
    p13.topk_w = topk_weights;
    p13.sched = ws.sched;
    p13.n_stages = prefill_stages((int)E, max_smem_optin());
#ifdef W4A16_DIAGNOSTICS
    if (const char* tr = getenv("W4A16_PREFILL_TRACE")) p13.trace = (long long*)strtoull(tr, nullptr, 0);
#endif
    PrefillParams p2 = p13;
    p2.trace = nullptr;
#ifdef W4A16_DIAGNOSTICS
    if (getenv("W4A16_PREFILL_TRACE_W2") != nullptr) {
      p2.trace = p13.trace;
      p13.trace = nullptr;
    }
#endif
    p2.w = (const uint8_t*)w2_rep;
    p2.s = (const uint8_t*)s2_rep;
    p2.n_rowtiles = (int)(H / 16);
    p2.n_chunks = (int)(I / 64);
    p2.x = ws.inter;
    p2.x_ld = I;
    p2.x_row_div = 1;
    p2.partial = (__nv_bfloat16*)ws.partial;  // bf16 partials in the fp32 partial region
    err = launch_prefill_w13(p13, sm_count(), st);
    if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_forward/prefill w13");
    mark_stage(2, st);
    err = launch_prefill_w2(p2, map, (int)M, (int)topk, (int)H, (__nv_bfloat16*)out, sm_count(), st);
    if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_forward/prefill w2");
    mark_stage(3, st);
    return kOk;
  }

  const RouteView rt{ws.sorted, ws.offsets, ws.counts, ws.active, ws.num_active, ws.tok_valid};
  const int64_t max_active = n_tok < E ? n_tok : E;
  const double avg_per_expert = (double)n_tok / (double)max_active;
  const int ng = avg_per_expert <= 2.0 ? 1 : (avg_per_expert <= 6.0 ? 2 : 4);
  const int sms = sm_count();

  // 2) w13 + SiLU(gate)*up -> inter[slot, I]
  GemvParams g1{};
  g1.w = (const uint4*)w13_rep;
  g1.s = (const uint2*)s13_rep;
  g1.n_rowtiles = (int)(2 * I / 16);
  g1.n_chunks = (int)(H / 64);
  g1.x = (const __nv_bfloat16*)hidden;
  g1.x_ld = hidden_ld;
  g1.x_row_div = (int)topk;
  g1.rt = rt;
  g1.topk = (int)topk;
  g1.items_per_expert = (int)(I / 16);
  g1.inter = ws.inter;
  g1.I = (int)I;
  g1.map = map;
  {
    const int64_t items = max_active * g1.items_per_expert;
    const int64_t cap = (int64_t)sms * gemv_blocks_per_sm(0, ng);
    const int grid = (int)(items < cap ? items : cap);
    err = launch_gemv(g1, 0, ng, grid, st);
    if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_forward/w13");
  }
  mark_stage(2, st);

  // 3) w2 * router weight, fused deterministic top-k sum -> out[M, H]
  GemvParams g2{};
  g2.w = (const uint4*)w2_rep;
  g2.s = (const uint2*)s2_rep;
  g2.n_rowtiles = (int)(H / 16);
  g2.n_chunks = (int)(I / 64);
  g2.x = ws.inter;
  g2.x_ld = I;
  g2.x_row_div = 1;
  g2.rt = rt;
  g2.topk = (int)topk;
  g2.items_per_expert = (int)(H / 32);
  g2.partial = ws.partial;
  g2.H = (int)H;
  g2.topk_w = topk_weights;
  g2.counters = ws.counters;
  g2.out = (__nv_bfloat16*)out;
  g2.map = map;
  {
    const int64_t items = max_active * g2.items_per_expert;
    const int64_t cap = (int64_t)sms * gemv_blocks_per_sm(1, ng);
    const int grid = (int)(items < cap ? items : cap);
    err = launch_gemv(g2, 1, ng, grid, st);
    if (err != cudaSuccess) return cuda_fail(err, "w4a16_moe_forward/w2");
  }
  mark_stage(3, st);
  return kOk;
}

}  // extern "C"
