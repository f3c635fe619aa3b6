/*
 * latchmoe_b200.h -- C ABI of liblatchmoe_b200.so, the B200 (sm_100a) data path of the
 * slot-bank MoE layer: router -> expert histogram -> pair grouping (permute) -> grouped
 * gate_up GEMM with fused SiLU*mul -> grouped down GEMM -> weighted top-k combine, plus the
 * host->device expert staging copy.
 *
 * Conventions shared by every entry point
 *   - All tensor arguments are raw DEVICE pointers unless the parameter name ends in
 *     `_host`. bf16 tensors are passed as `uint16_t*` (raw bf16 bit patterns).
 *   - `stream` is a cudaStream_t passed as `void*` (NULL = legacy default stream).
 *   - Every function returns LM_OK (0) or a negative LM_ERR_* code. No C++ exception
 *     crosses the ABI. On error `lm_last_error()` returns a message for this thread.
 *   - The library never allocates device memory on the hot path: the caller owns and
 *     pre-allocates every buffer (slot banks, permute/offset tables, scratch). Captured
 *     CUDA graphs may therefore replay these launches as long as the buffers stay put.
 *   - `err_word` (int32, device) receives the first device-side error code
 *     (LM_DEVERR_*); the host reads it outside graph capture. Kernels never trap: an
 *     out-of-range expert id or an unmapped expert is recorded and the pair is skipped,
 *     and every spin-wait is bounded.
 *
 * The reference (vllm_moe_offload_ascend) ships no native code; each entry point below
 * replaces a device operation that its Python call sites delegate to the Ascend stack.
 * The "Replaces" line names that call site (file:line within the reference project).
 */
#ifndef LATCHMOE_B200_H
#define LATCHMOE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LM_ABI_VERSION 1

#define LM_OK 0
#define LM_ERR_INVALID_ARGUMENT (-1)
#define LM_ERR_CUDA (-2)
#define LM_ERR_UNSUPPORTED (-3)
#define LM_ERR_DEVICE (-4)

/* Device-side error codes written to `err_word` (first error wins). */
#define LM_DEVERR_NONE 0
#define LM_DEVERR_BAD_EXPERT_ID 1   /* top-k id outside [0, num_experts) */
#define LM_DEVERR_UNMAPPED_EXPERT 2 /* expert routed but its group/slot entry is -1 */
#define LM_DEVERR_WAIT_TIMEOUT 3    /* a bounded mbarrier wait gave up */
#define LM_DEVERR_BAD_GROUP 4       /* group table inconsistent with the pair table */

/* Scoring functions accepted by lm_route_topk (reference `scoring_func`). */
#define LM_SCORING_SOFTMAX 0
#define LM_SCORING_SIGMOID 1

/* Staging copy directions accepted by lm_stage_copy. */
#define LM_COPY_H2D 1
#define LM_COPY_D2D 3

/* Weight sources in lm_slot_plan's per-group table (see lm_slot_plan). */
#define LM_SRC_MISS 0x40000000 /* flag: host store row, written through into the slot */
#define LM_SRC_HOST (-2)       /* host store row, not cached (working set > slots) */

/* ABI version (LM_ABI_VERSION of the built library). */
int lm_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* lm_last_error(void);

/*
 * K1 router: scores(logits) -> (optional grouped) top-k -> optional renormalisation
 * w / max(sum w, FLT_EPSILON) -> x routed_scaling_factor -> cast to bf16.
 * Selection ties go to the lower expert id. Softmax/sigmoid are monotone, so without a
 * correction bias the selection runs on the logits themselves (exact on the inputs).
 * logits [T, E] fp32 row-major; topk_weights_bf16 [T, k] (required); topk_weights_f32
 * [T, k] (optional, may be NULL); topk_ids [T, k] int32. E <= 256, k <= 32.
 * e_score_correction_bias [E] fp32 or NULL. num_expert_group/topk_group <= 1 disable
 * group-limited selection.
 * Replaces: ops/fused_moe/moe_router_op.py:98-124 (select_experts) and the CANN gating
 * fallback patches/patch_fused_moe.py:597-637.
 */
int lm_route_topk(const float* logits, int64_t num_tokens, int32_t num_experts,
                  int32_t top_k, int32_t scoring_func, int32_t renormalize,
                  float routed_scaling_factor, const float* e_score_correction_bias,
                  int32_t num_expert_group, int32_t topk_group,
                  uint16_t* topk_weights_bf16, float* topk_weights_f32,
                  int32_t* topk_ids, void* stream);

/*
 * K1 router with the fused mix-placement shared suffix: the same routed selection as
 * lm_route_topk over the num_experts routed experts, written as rows of top_k + num_shared
 * entries: the routed top-k, then the shared experts' logical ids num_experts ..
 * num_experts + num_shared - 1 with weight 1 (the slot bank's pinned suffix serves them).
 * topk_weights_bf16 / topk_weights_f32 / topk_ids are [T, top_k + num_shared];
 * top_k + num_shared <= 32.
 * Replaces: ops/fused_moe/moe_router_op.py:72-125 with mix_placement=True (select_experts
 * appending num_shared_experts pairs per token, moe_router_op.py:152-161).
 */
int lm_route_topk_shared(const float* logits, int64_t num_tokens, int32_t num_experts,
                         int32_t top_k, int32_t scoring_func, int32_t renormalize,
                         float routed_scaling_factor, const float* e_score_correction_bias,
                         int32_t num_expert_group, int32_t topk_group, int32_t num_shared,
                         uint16_t* topk_weights_bf16, float* topk_weights_f32,
                         int32_t* topk_ids, void* stream);

/*
 * K1 + K3 for a decode-sized call in one launch: the routing of lm_route_topk_shared
 * (num_shared may be 0) followed by the grouping of lm_build_groups over the
 * num_tokens * (top_k + num_shared) <= 512 pairs with expert_to_group [num_experts_total],
 * num_groups groups. Outputs are identical to the two calls. For a layer whose experts are
 * read in place, where the grouping does not depend on staging.
 */
int lm_route_group_small(const float* logits, int64_t num_tokens, int32_t num_experts,
                         int32_t top_k, int32_t scoring_func, int32_t renormalize,
                         float routed_scaling_factor, const float* e_score_correction_bias,
                         int32_t num_expert_group, int32_t topk_group, int32_t num_shared,
                         uint16_t* topk_weights_bf16, float* topk_weights_f32,
                         int32_t* topk_ids, int32_t num_experts_total,
                         const int32_t* expert_to_group, int32_t num_groups,
                         int32_t* group_offsets, int32_t* pair_to_row, int32_t* row_to_pair,
                         int32_t* err_word, void* stream);

/*
 * K2 active-expert histogram: counts[e] = #pairs routed to expert e (counts is
 * overwritten). Invalid ids set LM_DEVERR_BAD_EXPERT_ID in err_word (may be NULL).
 * Replaces: ops/fused_moe/moe_offload_stage_op.py:297-302,474-508 (D2H of all top-k ids
 * + host counting) and moe_offload/phase_split.py:479-492.
 */
int lm_expert_histogram(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                        int32_t* counts, int32_t* err_word, void* stream);

/*
 * K9a canonical wave plan on the device (one CTA) from the histogram `counts` [E]:
 * active experts sorted by (-count, id), ceil(U/S) waves, each expert into the least-loaded
 * wave with room (lowest index on ties), members ordered by id; groups numbered wave by wave.
 * Outputs: expert_to_group [E] (-1 inactive), group_bank_row [E] (entries 0..U-1: the
 * expert id when bank_row_mode == 0 -- experts read in place from an [E, ...] bank -- or
 * the position inside its wave when bank_row_mode == 1 -- positional stage-bank slots),
 * wave_offsets [E+1] (group range of wave w = [wave_offsets[w], wave_offsets[w+1])) and
 * num_waves [1]. E <= 1024.
 * Replaces: moe_offload/phase_split.py:495-555 (plan_balanced_b2_waves) run on the host
 * after the D2H of every top-k id (patches/patch_fused_moe.py:2518-2546).
 */
int lm_plan_waves(const int32_t* counts, int32_t num_experts, int32_t num_slots,
                  int32_t bank_row_mode, int32_t* expert_to_group, int32_t* group_bank_row,
                  int32_t* wave_offsets, int32_t* num_waves, void* stream);

/* Scratch (int32 elements) lm_build_groups needs for `num_pairs` pairs and `num_groups`. */
int64_t lm_build_groups_scratch_elems(int64_t num_pairs, int32_t num_groups);

/*
 * K4/K9 pair grouping (stable counting sort): pair p = t*k + j goes to group
 * g = expert_to_group[topk_ids[p]]. Rows of group g are [group_offsets[g],
 * group_offsets[g+1]) and keep the original flat pair order inside the group.
 * Outputs: group_offsets [G+1], pair_to_row [P] (row of pair p, -1 if unmapped),
 * row_to_pair [P] (pair of row r; rows past group_offsets[G] are left untouched).
 * With expert_to_group = log2phy this is the decode slot remap; with the wave table it is
 * the multi-wave pair planner.
 * Replaces: moe_offload/slot_mapping.py:116-141 (log2phy[topk_ids]), the CANN
 * npu_moe_init_routing_v2 call patches/patch_fused_moe.py:645-711, and
 * moe_offload/phase_split.py:1224-1385 (build_b2_device_wave_microbatch_plans).
 */
int lm_build_groups(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                    const int32_t* expert_to_group, int32_t num_groups,
                    int32_t* group_offsets, int32_t* pair_to_row, int32_t* row_to_pair,
                    int32_t* scratch, int64_t scratch_elems, int32_t* err_word,
                    void* stream);

/*
 * lm_build_groups without caller-owned scratch, for callers that cannot allocate device
 * memory themselves: a host that has already handed all free HBM to its own pool (a
 * serving engine sizing its KV cache to fill the card), or a foreign-language binding
 * that has no device allocator. Same inputs, outputs and results as lm_build_groups; the
 * scratch lives in one static device array of LM_NOALLOC_GROUP_SCRATCH_ELEMS int32 (512 KiB)
 * that every GPU loading this library keeps until the process exits. Calls needing more
 * (lm_build_groups_scratch_elems(num_pairs, num_groups) > the limit, e.g. more than
 * 262144 pairs at 128 groups) return LM_ERR_INVALID_ARGUMENT. The first call on a device
 * looks up the array's device address with that device current; make that first call
 * before any stream capture. All calls on a device share its array and the array keeps
 * the last call's contents, so calls that overlap on the GPU (for example on two streams
 * of one device) race and must be ordered by the caller. The passes write every scratch
 * entry they later read, so nothing needs clearing between calls. No cudaMalloc, cudaFree
 * or allocating library routine is used.
 * Has no counterpart in the reference (its grouping runs inside the Ascend stack).
 */
#define LM_NOALLOC_GROUP_SCRATCH_ELEMS 131072
int lm_build_groups_noalloc(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                            const int32_t* expert_to_group, int32_t num_groups,
                            int32_t* group_offsets, int32_t* pair_to_row, int32_t* row_to_pair,
                            int32_t* err_word, void* stream);

/*
 * Row gather: x_perm[r, :] = hidden[row_to_pair[r] / top_k, :] for r < num_rows.
 * hidden [T, H] bf16, x_perm [num_rows, H] bf16; H % 8 == 0.
 * Replaces: the token-permute half of npu_moe_init_routing_v2
 * (patches/patch_fused_moe.py:688-702).
 */
int lm_permute_rows(const uint16_t* hidden, int32_t hidden_size, const int32_t* row_to_pair,
                    int32_t top_k, int64_t num_rows, uint16_t* x_perm, void* stream);

/*
 * Grouped expert MLP over groups [group_begin, group_end).
 * Weights live in a "bank": w13_bank [bank_rows, 2I, H] (rows 0..I-1 = gate, I..2I-1 = up,
 * K-major) and w2_bank [bank_rows, H, I] (K-major); group g reads bank row
 * group_bank_row[g]. x_perm [R, H] bf16 (rows in group order), act [R, I] bf16 (written),
 * y_perm [R, H] bf16 (written). R = total rows (= group_offsets[num_groups]).
 *   act[r, j]  = silu(x_r . w13[j]) * (x_r . w13[I + j])    (fp32 accumulate)
 *   y_perm[r]  = act_r . w2^T                                (fp32 accumulate)
 * lm_moe_mlp_decode: bandwidth-bound GEMV path for small groups (reads hidden rows through
 *   row_to_pair directly; x_perm is not needed). Requires H % 32 == 0, I % 32 == 0.
 * lm_moe_mlp_prefill: tcgen05/TMEM grouped GEMM fed by TMA (128x256x64 tiles, persistent
 *   CTAs). Requires H % 256 == 0, I % 128 == 0, 16-byte aligned bases.
 * Replaces: the two npu_grouped_matmul calls and npu_swiglu inside the host
 * unified_apply_mlp (patches/patch_fused_moe.py:4249-4302, moe_offload/phase_split.py:2167).
 */
int lm_moe_mlp_decode(const uint16_t* hidden, int32_t top_k, const int32_t* row_to_pair,
                      const int32_t* group_offsets, const int32_t* group_bank_row,
                      int32_t group_begin, int32_t group_end, int32_t max_rows_per_group,
                      const uint16_t* w13_bank, const uint16_t* w2_bank, int64_t bank_rows,
                      int32_t hidden_size, int32_t intermediate_size,
                      uint16_t* act, uint16_t* y_perm, int32_t* err_word, void* stream);

/*
 * The persistent decode kernel keeps its work queue in one of 16 counter sets per device, one
 * per stream. A set moves to another stream once its stream's last eager launch has
 * completed; a set used inside a stream capture stays with that stream. When no set can be
 * freed, the launch runs the two-kernel decode path (same outputs) and is counted here.
 * Reports the current device's sets in use, those held by captures, sets moved so far and
 * launches that fell back (any pointer may be NULL).
 */
int lm_decode_counter_sets(int32_t* in_use, int32_t* pinned, int64_t* recycled,
                           int64_t* fallbacks);

int lm_moe_mlp_prefill(const uint16_t* x_perm, int64_t total_rows,
                       const int32_t* group_offsets, const int32_t* group_bank_row,
                       int32_t group_begin, int32_t group_end,
                       const uint16_t* w13_bank, const uint16_t* w2_bank, int64_t bank_rows,
                       int32_t hidden_size, int32_t intermediate_size,
                       uint16_t* act, uint16_t* y_perm, int32_t* err_word, void* stream);

/*
 * lm_moe_mlp_prefill_rows: the same MLP with the down GEMM's output row r stored at
 * y_row_ptrs[r] (a device array of total_rows 16-byte-aligned row pointers, which may address
 * another GPU's memory mapped into this process) instead of y_perm[r]. The kernel ends with a
 * system-scope fence, so a flag raised by a later kernel in the stream orders those stores.
 */
int lm_moe_mlp_prefill_rows(const uint16_t* x_perm, int64_t total_rows,
                            const int32_t* group_offsets, const int32_t* group_bank_row,
                            int32_t group_begin, int32_t group_end,
                            const uint16_t* w13_bank, const uint16_t* w2_bank, int64_t bank_rows,
                            int32_t hidden_size, int32_t intermediate_size,
                            uint16_t* act, uint16_t* const* y_row_ptrs, int32_t* err_word,
                            void* stream);

/*
 * Multi-wave execution from a device wave plan (lm_plan_waves with bank_row_mode 1), with no
 * host step between the waves:
 *   lm_stage_wave_copy: expert e joins stage row expert_to_group[e] - wave_offsets[wave] when
 *     the plan put it in wave `wave` (rows of bytes_per_expert bytes; dst holds dst_rows rows;
 *     bases, strides and size multiples of 16 bytes); nothing happens for wave >= *num_waves.
 *   lm_moe_mlp_prefill_wave: lm_moe_mlp_prefill over the groups of wave `wave`
 *     [wave_offsets[wave], wave_offsets[wave + 1]) read on the device (none when
 *     wave >= *num_waves; at most 256 groups).
 * A caller launches ceil(E / S) waves; the plan decides how many do any work.
 */
int lm_stage_wave_copy(void* dst, int64_t dst_row_stride, int32_t dst_rows, const void* src,
                       int64_t src_row_stride, int32_t num_experts, int64_t bytes_per_expert,
                       const int32_t* expert_to_group, const int32_t* wave_offsets,
                       const int32_t* num_waves, int32_t wave, void* stream);
int lm_moe_mlp_prefill_wave(const uint16_t* x_perm, int64_t total_rows,
                            const int32_t* group_offsets, const int32_t* group_bank_row,
                            const int32_t* wave_offsets, const int32_t* num_waves, int32_t wave,
                            const uint16_t* w13_bank, const uint16_t* w2_bank, int64_t bank_rows,
                            int32_t hidden_size, int32_t intermediate_size, uint16_t* act,
                            uint16_t* y_perm, int32_t* err_word, void* stream);

/*
 * K8 weighted combine in the original flattened top-k pair order:
 *   out[t, :] = bf16( sum_{j<k} f32(topk_weights[t, j]) * f32(y_perm[pair_to_row[t*k+j], :]) )
 * accumulated in fp32 in j order (deterministic, no atomics). pair_to_row < 0 contributes 0.
 * Replaces: the single native token_combine after all waves
 * (patches/patch_fused_moe.py:3340-3366, moe_offload/phase_split.py:1765-1856).
 */
int lm_moe_combine(const uint16_t* y_perm, const int32_t* pair_to_row,
                   const uint16_t* topk_weights_bf16, int64_t num_tokens, int32_t top_k,
                   int32_t hidden_size, uint16_t* out, void* stream);

/*
 * Device-count variants, for a caller whose count is only known on the device (e.g. rows an
 * exchange has just received): each call covers min(max, *count_dev) pairs / rows / tokens,
 * read by the kernels, with buffers sized for max. Same results as the plain calls on that
 * many items; entries past the count are left as they are.
 * Replaces: nothing in the reference, which is single-device; these serve the owner side of
 * the expert-partitioned exchange (lm_ep_* below), keeping its received count on the device.
 */
int lm_build_groups_count(const int32_t* topk_ids, int64_t max_pairs,
                          const int32_t* num_pairs_dev, int32_t num_experts,
                          const int32_t* expert_to_group, int32_t num_groups,
                          int32_t* group_offsets, int32_t* pair_to_row, int32_t* row_to_pair,
                          int32_t* scratch, int64_t scratch_elems, int32_t* err_word,
                          void* stream);
int lm_permute_rows_count(const uint16_t* hidden, int32_t hidden_size,
                          const int32_t* row_to_pair, int32_t top_k, int64_t max_rows,
                          const int32_t* num_rows_dev, uint16_t* x_perm, void* stream);
/* Row gather through a second index, for rows another GPU wrote this call (read at L2):
 * x_perm[r, :] = src[pair_src[row_to_pair[r]], :] for r < min(max_rows, *num_rows_dev). */
int lm_permute_rows_gather_count(const uint16_t* src, int32_t hidden_size,
                                 const int32_t* row_to_pair, const int32_t* pair_src,
                                 int64_t max_rows, const int32_t* num_rows_dev, uint16_t* x_perm,
                                 void* stream);
int lm_moe_combine_count(const uint16_t* y_perm, const int32_t* pair_to_row,
                         const uint16_t* topk_weights_bf16, int64_t max_tokens,
                         const int32_t* num_tokens_dev, int32_t top_k, int32_t hidden_size,
                         uint16_t* out, void* stream);

/*
 * K10 expert staging: for i < n, copy bytes_per_expert bytes from
 * src + src_rows_host[i]*src_row_stride to dst + dst_rows_host[i]*dst_row_stride with
 * cudaMemcpyAsync on `stream`, coalescing runs where both row sequences are consecutive
 * into one copy. kind = LM_COPY_H2D (src is pinned host memory) or LM_COPY_D2D. A D2D copy
 * whose bases, strides and size are multiples of 16 bytes runs as one copy kernel per 64
 * rows instead. Returns the number of copies issued (cudaMemcpyAsync calls or kernel
 * launches, >= 0) or a negative error.
 * Replaces: moe_offload/transfer_engine.py:139-187,205-228,246-303 (load_many_async,
 * _copy_loads, _try_batch_view).
 */
int lm_stage_copy(void* dst, int64_t dst_row_stride, const void* src, int64_t src_row_stride,
                  const int32_t* src_rows_host, const int32_t* dst_rows_host, int32_t n,
                  int64_t bytes_per_expert, int32_t kind, void* stream);

/*
 * Device-side staging decision of one decode stage call (no device->host round trip).
 * State in device memory, persistent across calls, initialised by the caller once:
 * slot_owner [num_slots] int32 = -1, slot_last_used [num_slots] int64 = -1,
 * expert_slot [num_experts] int32 = -1, step_counter [1] int64 = 0.
 * From topk_ids [num_pairs] it marks the active experts and, when their count is at most
 * num_slots, assigns slots in ascending expert order: a resident expert's last-used step is
 * bumped; a missing one takes the first empty slot, else the slot with the least
 * (last_used, slot id) among those not assigned in this call; log2phy[e] = slot of every
 * active expert. It writes group_src [num_experts] (group = expert id): slot s for a hit,
 * s | LM_SRC_MISS for a miss (the MLP reads the host store and fills slot s), LM_SRC_HOST
 * when the working set exceeds the slots (the bank is then left untouched, as the reference's
 * multi-wave path leaves it), -1 for inactive experts. hit_miss_counts (int64 [2], may be
 * NULL) accumulates the hits and misses of the calls that assigned slots.
 * num_experts <= 8192, num_slots <= 1024.
 * Replaces: the stage seam's blocking D2H and Python allocation loop
 * (ops/fused_moe/moe_offload_stage_op.py:297-302, moe_offload/runtime.py:1636-1902,
 * moe_offload/slot_bank.py:211-232).
 */
int lm_slot_plan(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                 int32_t num_slots, int32_t* slot_owner, int64_t* slot_last_used,
                 int32_t* expert_slot, int64_t* step_counter, int32_t* log2phy,
                 int32_t* group_src, int64_t* hit_miss_counts, int32_t* err_word,
                 void* stream);

/*
 * Decode grouped MLP with the weight source per group taken from lm_slot_plan's table:
 * slot rows of w13_slots [num_slots, 2I, H] / w2_slots [num_slots, H, I], or rows
 * group_expert[g] of the pinned host store w13_host [num_experts, 2I, H] / w2_host
 * [num_experts, H, I] (read by the kernel over PCIe; for LM_SRC_MISS every loaded chunk is
 * also written into the slot). Same math and outputs as lm_moe_mlp_decode; at most 64 rows
 * per group (one weight pass). Requires H % 128 == 0, I % 64 == 0, 16-byte aligned bases,
 * host stores allocated as pinned memory.
 * Replaces: the H2D staging of missed experts (moe_offload/transfer_engine.py:139-187)
 * together with the grouped MLP (patches/patch_fused_moe.py:4249-4302).
 */
int lm_moe_mlp_decode_offload(const uint16_t* hidden, int32_t top_k,
                              const int32_t* row_to_pair, const int32_t* group_offsets,
                              const int32_t* group_src, const int32_t* group_expert,
                              int32_t group_begin, int32_t group_end, int32_t max_rows_per_group,
                              uint16_t* w13_slots, uint16_t* w2_slots, int32_t num_slots,
                              const uint16_t* w13_host, const uint16_t* w2_host,
                              int32_t num_experts, int32_t hidden_size,
                              int32_t intermediate_size, uint16_t* act, uint16_t* y_perm,
                              int32_t* err_word, void* stream);

/*
 * Expert-parallel exchange over peer memory (one process per GPU; no NCCL on the data path).
 * Each rank allocates one region (lm_ep_region_alloc, size lm_ep_region_bytes) and maps every
 * other rank's region (lm_ipc_get_handle -> exchange the 64-byte handles -> lm_ipc_open_handle).
 * peer_regions is a DEVICE array of `world` pointers (entry `rank` = the rank's own region).
 * cap = most routed pairs one source sends to one owner. epoch = a call counter, the same on
 * every rank and increasing by one per layer call (flags hold the last epoch seen). epoch 0
 * means the counter kept in the rank's own region instead: lm_ep_advance_epoch raises it on
 * the device at the start of each call, so a step captured in a CUDA graph gets a new epoch
 * on every replay (every rank advances once per call; do not mix the two forms on one
 * exchange).
 * Per layer call, in stream order on every rank:
 *   lm_ep_dispatch      pairs grouped by owner (pair_to_row / send_offsets from
 *                       lm_build_groups with expert -> owner); each pair's hidden row and
 *                       owner-local expert id go straight into the owner's region.
 *   (or lm_ep_dispatch_tokens: the same pair metadata, but each token's row is stored once
 *    per owner that holds any of its experts, at receive row rank * (cap / top_k) + its token
 *    slot; tok_slot [num_tokens * world] (-1: no pair there) and tok_count [world] are
 *    written on the device. Owners read rows through each pair's receive-row index, so the
 *    receive side is the same for both dispatches.)
 *   lm_ep_receive       waits for every source's dispatch (bounded), compacts the received rows
 *                       and ids into rows_out / ids_out; *total_out = their number (device).
 *   (local expert MLP, outputs written in received order at region + lm_ep_out_rows_offset)
 *   (or lm_ep_receive_index: the same wait, then only the received pairs' receive-area slots
 *    and ids in received order; the owner gathers its rows from the receive area itself,
 *    region + lm_ep_recv_rows_offset, with lm_permute_rows_gather_count, and writes the output
 *    row of received pair d to the int32 table at region + lm_ep_pair_rows_offset)
 *   (or the owner pushes: lm_ep_output_row_ptrs turns the grouped rows' received pairs
 *    (row_to_pair, *count_dev rows) into row pointers into each source's output area, block
 *    rank, at the pair's position, and lm_moe_mlp_prefill_rows stores the outputs there;
 *    the sources then combine with lm_ep_combine_local, which reads only their own region)
 *   lm_ep_signal_outputs  tells every source the outputs are there.
 *   lm_ep_combine       waits for every owner (bounded), reads each pair's output row from its
 *                       owner (row = the owner's pair-row table entry; lm_ep_receive writes
 *                       received order there) and reduces out[t] = sum_j w[t,j] * y[t,j] in
 *                       fp32, j in order.
 * done_counter: one device int32, zero before the first call. Waits that run out set
 * LM_DEVERR_WAIT_TIMEOUT; after a timed-out output wait lm_ep_combine reads nothing from the
 * owners and writes zero rows. num_tokens * top_k > cap is rejected with
 * LM_ERR_INVALID_ARGUMENT by lm_ep_dispatch and lm_ep_combine, and a pair whose position in
 * its owner's area falls outside [0, cap) is skipped and recorded as LM_DEVERR_BAD_GROUP.
 * Ranks must be on distinct GPUs.
 * Replaces: nothing in the reference, which is single-device
 * (patches/patch_fused_moe.py:4898-4914); the combine follows token_combine's order
 * (moe_offload/phase_split.py:1765-1856).
 */
int64_t lm_ep_region_bytes(int32_t world, int32_t cap, int32_t hidden_size);
int64_t lm_ep_out_rows_offset(int32_t world, int32_t cap, int32_t hidden_size);
int lm_ep_region_alloc(int64_t bytes, void** region);
int lm_ep_region_free(void* region);
int lm_ipc_get_handle(const void* region, void* handle_out /* 64 bytes */);
int lm_ipc_open_handle(const void* handle /* 64 bytes */, void** region_out);
int lm_ipc_close_handle(void* region);
int lm_ep_dispatch(const uint16_t* hidden, int64_t num_tokens, int32_t top_k,
                   int32_t hidden_size, const int32_t* topk_ids, int32_t experts_per_rank,
                   const int32_t* pair_to_row, const int32_t* send_offsets, int32_t rank,
                   int32_t world, void* const* peer_regions, int32_t cap, int64_t epoch,
                   int32_t* done_counter, int32_t* err_word, void* stream);
int lm_ep_dispatch_tokens(const uint16_t* hidden, int64_t num_tokens, int32_t top_k,
                          int32_t hidden_size, const int32_t* topk_ids,
                          int32_t experts_per_rank, const int32_t* pair_to_row,
                          const int32_t* send_offsets, int32_t rank, int32_t world,
                          void* const* peer_regions, int32_t cap, int64_t epoch,
                          int32_t* tok_slot, int32_t* tok_count, int32_t* done_counter,
                          int32_t* err_word, void* stream);
int lm_ep_receive(void* region, int32_t world, int32_t cap, int32_t hidden_size, int64_t epoch,
                  uint16_t* rows_out, int32_t* ids_out, int32_t* total_out, int32_t* err_word,
                  void* stream);
int lm_ep_receive_index(void* region, int32_t world, int32_t cap, int32_t hidden_size,
                        int64_t epoch, int32_t* slot_out, int32_t* ids_out, int32_t* total_out,
                        int32_t* err_word, void* stream);
int64_t lm_ep_recv_rows_offset(int32_t world, int32_t cap, int32_t hidden_size);
int64_t lm_ep_pair_rows_offset(int32_t world, int32_t cap, int32_t hidden_size);
int lm_ep_output_row_ptrs(void* region, int32_t world, int32_t cap, int32_t hidden_size,
                          int32_t rank, void* const* peer_regions, const int32_t* row_to_pair,
                          const int32_t* count_dev, int32_t max_rows, uint16_t** row_ptrs_out,
                          int32_t* err_word, void* stream);
int lm_ep_combine_local(const int32_t* topk_ids, const uint16_t* topk_weights_bf16,
                        int64_t num_tokens, int32_t top_k, int32_t hidden_size,
                        int32_t experts_per_rank, const int32_t* pair_to_row,
                        const int32_t* send_offsets, int32_t rank, int32_t world,
                        void* const* peer_regions, void* local_region, int32_t cap,
                        int64_t epoch, uint16_t* out, int32_t* err_word, void* stream);
/* Step figures on the device (int64 [4]): stats[0] += *total (pairs received), stats[1] +=
 * pairs kept local, stats[2] += rows the dispatch stored into other ranks (sum of tok_count
 * over the other ranks, or num_pairs - local when tok_count is NULL), stats[3] += num_pairs. */
int lm_ep_step_stats(const int32_t* total, const int32_t* send_offsets, const int32_t* tok_count,
                     int64_t num_pairs, int32_t rank, int32_t world, int64_t* stats,
                     void* stream);
int lm_ep_advance_epoch(void* region, int32_t world, int32_t cap, int32_t hidden_size,
                        void* stream);
int lm_ep_signal_outputs(void* const* peer_regions, int32_t rank, int32_t world, int32_t cap,
                         int32_t hidden_size, int64_t epoch, void* stream);
int lm_ep_combine(const int32_t* topk_ids, const uint16_t* topk_weights_bf16,
                  int64_t num_tokens, int32_t top_k, int32_t hidden_size,
                  int32_t experts_per_rank, const int32_t* pair_to_row,
                  const int32_t* send_offsets, int32_t rank, int32_t world,
                  void* const* peer_regions, void* local_region, int32_t cap, int64_t epoch,
                  uint16_t* out, int32_t* err_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LATCHMOE_B200_H */
