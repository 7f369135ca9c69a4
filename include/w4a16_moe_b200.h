/*
 * C ABI of the B200 (sm_100a) W4A16 grouped-MoE library.
 *
 * Every entry point takes raw device pointers, 64-bit sizes and a CUDA stream
 * passed as `void*` (a cudaStream_t; NULL = legacy default stream), launches
 * asynchronously on that stream and returns a status:
 *   0 = ok, 1 = invalid argument, 2 = unsupported shape, 3 = CUDA error.
 * On a nonzero status w4a16_last_error() returns a message for the calling
 * thread.  No entry point allocates device memory, synchronises the device or
 * copies between host and device, so all of them can be captured in a CUDA
 * graph once the workspace exists.
 *
 * Tensors (all row-major, contiguous unless a leading dimension is given):
 *   bf16 values are passed as their 16-bit patterns.
 *   Packed int4 weights use the vLLM / compressed-tensors post-load layout:
 *   (E, N_out, K/2) uint8, byte j of a row = element 2j (low nibble) and
 *   2j+1 (high nibble), stored value = q + 8, q in [-8, 7].
 */
#ifndef W4A16_MOE_B200_H_
#define W4A16_MOE_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define W4A16_API __attribute__((visibility("default")))
#else
#define W4A16_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Message for the last failing call on this thread ("" if none). */
W4A16_API const char* w4a16_last_error(void);

/* Library ABI version (major*100 + minor). */
W4A16_API int w4a16_version(void);

/*
 * Profiling hook (no reference counterpart): for the calling thread, have
 * w4a16_moe_forward record events[i] (cudaEvent_t handles) on its stream at
 * stage boundaries: 0 before routing, 1 after routing, 2 after the w13 GEMM,
 * 3 after the w2 GEMM.  Works inside CUDA-graph capture (external event
 * records).  n_events = 0 disables it.
 */
W4A16_API int w4a16_set_stage_events(void* const* events, int n_events);

/*
 * Path selection for the calling thread (no reference counterpart; used by
 * tests to cover every implementation): 0 = automatic (staged fused
 * persistent kernel for M*topk <= 4096, tcgen05 prefill kernels or the
 * CUDA-core general path otherwise), 1 = always the general path, 2 = the
 * tcgen05 prefill kernels wherever their shape rules allow, 3 = the
 * direct-streaming decode kernel wherever it applies.
 */
W4A16_API int w4a16_set_path(int path);

/*
 * Reads and clears the error bits the fused kernel records in a workspace
 * (0 = none; bit 0/1 = pipeline wait timed out, bit 2 = cross-CTA wait timed
 * out).  Synchronises `stream`; diagnostic use only.
 */
W4A16_API int w4a16_moe_read_status(const void* workspace, int64_t M, int64_t topk, int64_t E,
                                    int64_t H, int64_t I, int32_t* status_out, void* stream);

/*
 * Length P of sorted_token_ids for moe_align_block_size:
 * roundup(n_tok + num_experts*(block_size-1), block_size).
 * Replaces the sizing in kernels/w4a16_moe.py:153-157 (_align_workspace).
 */
W4A16_API int64_t w4a16_align_buffer_len(int64_t n_tok, int64_t num_experts, int64_t block_size);

/*
 * Expert-sorted, block-padded slot order.  Bit-exact with the reference's
 * moe_align_block_size (kernels/w4a16_moe.py:187-290):
 *   sorted_token_ids [P]            int32, padding = M*topk
 *   expert_ids       [P/block_size] int32, -1 past num_tokens_post_padded
 *   num_tokens_post_padded [1]      int32
 * topk_ids: [M, topk] int32 (ids_is_int64 = 0) or int64 (1).
 * num_experts <= 1024.
 */
W4A16_API int w4a16_moe_align(const void* topk_ids, int ids_is_int64, int64_t M, int64_t topk,
                    int64_t num_experts, int64_t block_size, int32_t* sorted_token_ids,
                    int32_t* expert_ids, int32_t* num_tokens_post_padded, void* stream);

/*
 * Same outputs as w4a16_moe_align, with caller-provided scratch that lets
 * large inputs run as one multi-CTA cooperative kernel instead of one CTA
 * (no reference counterpart).  scratch: w4a16_moe_align_scratch_bytes()
 * bytes, 256-byte aligned, zero-filled once before its first use and left
 * clean by every call; calls sharing one scratch must be stream-ordered.
 * With scratch == NULL or a size of 0 this is w4a16_moe_align.
 */
W4A16_API int64_t w4a16_moe_align_scratch_bytes(int64_t n_tok, int64_t num_experts);
W4A16_API int w4a16_moe_align_ex(const void* topk_ids, int ids_is_int64, int64_t M, int64_t topk,
                    int64_t num_experts, int64_t block_size, int32_t* sorted_token_ids,
                    int32_t* expert_ids, int32_t* num_tokens_post_padded, void* scratch,
                    int64_t scratch_bytes, void* stream);

/*
 * Status of the multi-CTA align kernels that used `scratch` (no reference
 * counterpart).  *status_out receives the error bits of the calls since the
 * last query (bit 16: the grid barrier timed out; that call wrote no
 * outputs).  The query also resets the scratch's barrier words, so a scratch
 * whose call timed out is usable again afterwards.  Synchronises `stream`.
 */
W4A16_API int w4a16_moe_align_read_status(void* scratch, int32_t* status_out, void* stream);

/*
 * Test hook for the bounded device waits (no reference counterpart): mode 1
 * makes the calling thread's next multi-CTA align launches withhold one CTA's
 * arrival at the grid barrier and wait only ~10 us, so the wait runs out and
 * the timeout is reported as status; mode 2 makes the fused decode kernel's
 * CTA 0 publish none of its w13 items and the w2 items wait only ~10 us for
 * them, so those waits run out, the call finishes with wrong values and
 * w4a16_moe_read_status reports bit 4; mode 0 restores normal operation.
 */
W4A16_API int w4a16_set_wait_test(int mode);

/*
 * Load-time weight transform into this library's fragment-major layout.
 * Replaces repack_weights (kernels/w4a16_moe.py:63-116).
 *   w_q     (E, N_out, K/2) uint8        scales (E, N_out, K/group_size) bf16
 *   w_rep   (E, N_out/16, K/64, 512) u8  s_rep  (E, N_out/16, K/64, 32) bf16
 * Requires N_out % 16 == 0, K % 64 == 0, group_size % 32 == 0, K % group_size == 0.
 */
W4A16_API int w4a16_repack(const uint8_t* w_q, const void* scales, int64_t E, int64_t N_out, int64_t K,
                 int64_t group_size, uint8_t* w_rep, void* s_rep, void* stream);

/*
 * Same output as w4a16_repack, read straight from the checkpoint's
 * compressed-tensors pack-quantized tensors as vLLM's create_weights stores
 * them (is_transposed=True): w_packed int32 (E, K/8, N_out), code j of a word
 * at bits 4j (stored value q + 8); scales bf16 (E, K/group, N_out).  Replaces
 * the transpose(1, 2).contiguous().view(uint8) + repack_weights of the load
 * path (integration/apply.py:100-105 and kernels/w4a16_moe.py:63-116 in the
 * reference) with one launch pair and no intermediate copy.
 */
W4A16_API int w4a16_repack_checkpoint(const int32_t* w_packed, const void* scales, int64_t E, int64_t N_out,
                    int64_t K, int64_t group_size, uint8_t* w_rep, void* s_rep, void* stream);

/*
 * Router: per token, the top-k experts of fp32 logits [M, E] (row stride
 * logits_ld) in descending logit order (ties: lower id) and the softmax of
 * those k logits -- the routing the reference benchmarks
 * (bench/bench_moe.py:225-231: torch.topk then torch.softmax over the k
 * values).  topk_weights [M, topk] fp32, topk_ids [M, topk] int32;
 * E <= 1024, topk <= 32.  Logits must be finite.
 */
W4A16_API int w4a16_topk_softmax(const float* logits, int64_t M, int64_t E, int64_t logits_ld, int64_t topk,
                    float* topk_weights, int32_t* topk_ids, void* stream);

/* Bytes of workspace w4a16_moe_forward needs for this shape. */
W4A16_API int64_t w4a16_moe_workspace_size(int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I);

/*
 * Fused W4A16 MoE layer: routing align -> w13 GEMM + SiLU(gate)*up -> w2 GEMM
 * with the router-weighted top-k sum fused in.
 * Replaces fused_experts_w4a16 (kernels/w4a16_moe.py:678-909).
 *
 *   hidden        [M, H] bf16, row stride hidden_ld elements
 *   w13_rep/s13   repacked (E, 2I/16, H/64, ...) gate rows [0,I), up rows [I,2I)
 *   w2_rep/s2     repacked (E, H/16, I/64, ...)
 *   topk_weights  [M, topk] fp32          topk_ids [M, topk] int32 / int64
 *   expert_map    nullable [global_num_experts] int32: global id -> local id
 *                 in [0, E) or -1 (slot skipped), the vLLM EP convention
 *   out           [M, H] bf16 (fully written; rows with no local slot are 0)
 *   workspace     >= w4a16_moe_workspace_size bytes, 256-byte aligned, ZERO-
 *                 FILLED BEFORE ITS FIRST USE; every call leaves it reusable.
 *                 Calls sharing one workspace must be stream-ordered.
 * Requires H % 64 == 0, I % 64 == 0, E <= 1024.
 */
W4A16_API int w4a16_moe_forward(const void* hidden, int64_t M, int64_t H, int64_t hidden_ld,
                      const void* w13_rep, const void* s13_rep, const void* w2_rep,
                      const void* s2_rep, int64_t E, int64_t I, const float* topk_weights,
                      const void* topk_ids, int ids_is_int64, int64_t topk,
                      const int32_t* expert_map, int64_t global_num_experts, void* out,
                      void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Allocation-free variant of w4a16_moe_forward (no counterpart in the
 * reference).  For callers that may not allocate device memory where they run
 * the layer (inside another framework's memory pool or allocator hooks, in
 * plug-in hosts that forbid allocation on the hot path, on initialisation or
 * error paths): same arguments minus the workspace, which is replaced by a
 * 16 MiB static device array inside this library (held on every GPU that
 * loads it, until exit).  Shapes needing a larger workspace are rejected with
 * status 2.  All calls on a device share the array: calls that may overlap on
 * the GPU race.  The first call on a device resolves the array's address
 * (cudaGetSymbolAddress) and should come before any stream capture.
 */
W4A16_API int w4a16_moe_forward_noalloc(const void* hidden, int64_t M, int64_t H, int64_t hidden_ld,
                                        const void* w13_rep, const void* s13_rep, const void* w2_rep,
                                        const void* s2_rep, int64_t E, int64_t I,
                                        const float* topk_weights, const void* topk_ids,
                                        int ids_is_int64, int64_t topk, const int32_t* expert_map,
                                        int64_t global_num_experts, void* out, void* stream);

/* Size in bytes of the static scratch array behind w4a16_moe_forward_noalloc. */
W4A16_API int64_t w4a16_moe_noalloc_max_workspace(void);

/*
 * Status word of the last w4a16_moe_forward_noalloc call of this shape on the
 * current device (no reference counterpart): bits of bounded device waits
 * that ran out, as w4a16_moe_read_status reports them; reading clears them.
 * Synchronises `stream`.
 */
W4A16_API int w4a16_moe_noalloc_read_status(int64_t M, int64_t topk, int64_t E, int64_t H, int64_t I,
                                            int32_t* status_out, void* stream);

/*
 * Expert-parallel token exchange (no counterpart in the reference, which runs
 * on one GPU; these serve vLLM's expert_map / global_num_experts contract).
 * Rank r of G owns experts [r*E/G, (r+1)*E/G); E % G == 0.
 *
 * w4a16_ep_plan: per source token, the ranks owning any of its top-k experts.
 *   send_counts [G], send_offsets [G+1] (rank-major send order, tokens
 *   ascending inside a rank), send_tok [<= M*G] (token of each send row),
 *   tok_row [M*G] (send row of (token m, rank r) or -1).
 * w4a16_ep_pack: gathers hidden rows and their routing into send order:
 *   x_send [n_send, H] bf16, meta_send [n_send, 2*topk] int32 = top-k ids
 *   then the fp32 bit patterns of the top-k weights; n_send = send_offsets[G]
 *   is read on the device (buffers sized M*G rows).
 * w4a16_ep_combine: out[m] = bf16(sum over r ascending of back[tok_row[m,r]])
 *   in fp32; rows with no destination are zero.  back [n_send, H] bf16.
 */
W4A16_API int w4a16_ep_plan(const void* topk_ids, int ids_is_int64, int64_t M, int64_t topk,
                    int64_t num_experts, int64_t n_ranks, int32_t* send_counts,
                    int32_t* send_offsets, int32_t* send_tok, int32_t* tok_row, void* stream);
W4A16_API int w4a16_ep_pack(const void* hidden, int64_t hidden_ld, const void* topk_ids, int ids_is_int64,
                    const float* topk_weights, int64_t M, int64_t topk, int64_t H, int64_t n_ranks,
                    const int32_t* send_offsets, const int32_t* send_tok, void* x_send,
                    int32_t* meta_send, void* stream);
W4A16_API int w4a16_ep_combine(const void* back, const int32_t* tok_row, int64_t M, int64_t n_ranks,
                    int64_t H, void* out, void* stream);

/*
 * Fixed-capacity dispatch (no reference counterpart): plan + pack into G
 * blocks of `capacity` rows (capacity >= M, equal on every rank), so the
 * exchange is one all-to-all with equal splits and needs no host read of the
 * counts.  Block r: the tokens routed to rank r in ascending order, then
 * padding rows whose top-k ids are -1.  Row i of send_rows (row_stride bf16
 * elements, row_stride >= H + 4*topk, a multiple of 8) = [hidden | top-k ids
 * int32 | top-k weights fp32 bits | zeros].  send_counts [G]: valid rows per
 * block; send_tok [G*capacity]: token of each valid row; tok_row [M*G]: row
 * of (token m, rank r) or -1 (for w4a16_ep_combine on the returned rows).
 */
W4A16_API int w4a16_ep_dispatch_fixed(const void* hidden, int64_t hidden_ld, const void* topk_ids,
                    int ids_is_int64, const float* topk_weights, int64_t M, int64_t topk,
                    int64_t num_experts, int64_t H, int64_t n_ranks, int64_t capacity,
                    int64_t row_stride, void* send_rows, int32_t* send_counts, int32_t* send_tok,
                    int32_t* tok_row, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* W4A16_MOE_B200_H_ */
