// Device-side staging decision for decode: the slot-bank allocation of one stage call, run on
// the GPU so that a decode step needs no device->host round trip per layer (and can be
// captured whole in a CUDA graph).
//
// Semantics follow the reference allocator (moe_offload/slot_bank.py:211-232 allocate_for,
// driven by runtime.py:1636-1902 prepare_fixed_slot_plan_into_log2phy): slots still loading
// from the previous call are READY at the start of a call; the active experts are visited in
// ascending id order; a resident expert only has its last-used step bumped; a missing
// expert takes the first EMPTY slot, else the READY slot with the least
// (last_used_step, slot_id) (slots allocated earlier in the same call are LOADING and not
// evictable); log2phy gets the slot of every active expert. When the working set exceeds the
// slots the reference runs the multi-wave path, which leaves the slot bank untouched; here the
// bank is left untouched too and the experts without a slot are read from the host store.
//
// State (device memory, per layer, persistent across calls): slot_owner[S] (expert or -1),
// slot_last_used[S], expert_slot[E] (slot or -1), step counter. The per-group source table
// tells the streaming MLP where each active expert's weights come from:
//   s >= 0            : slot s (a hit)
//   s | LM_SRC_MISS   : host store row e, written through into slot s (a miss)
//   LM_SRC_HOST       : host store row e, not cached (working set larger than the slots)
//   -1                : inactive
#include "lm_common.cuh"

namespace lm {
namespace {

constexpr int kPlanMaxExpertsSlots = 8192;
constexpr int kPlanMaxSlots = 1024;

__global__ void __launch_bounds__(32)
    slot_plan_kernel(const int32_t* __restrict__ ids, int64_t num_pairs, int num_experts,
                     int num_slots, int32_t* __restrict__ slot_owner,
                     long long* __restrict__ slot_last, int32_t* __restrict__ expert_slot,
                     long long* __restrict__ step_counter, int32_t* __restrict__ log2phy,
                     int32_t* __restrict__ group_src, long long* __restrict__ hit_miss,
                     int32_t* __restrict__ err_word) {
  __shared__ uint8_t s_active[kPlanMaxExpertsSlots];
  __shared__ uint8_t s_loading[kPlanMaxSlots];
  const int lane = threadIdx.x;
  for (int e = lane; e < num_experts; e += 32) {
    s_active[e] = 0;
    group_src[e] = -1;
  }
  for (int s = lane; s < num_slots; s += 32) s_loading[s] = 0;
  __syncwarp();
  for (int64_t p = lane; p < num_pairs; p += 32) {
    const int e = ids[p];
    if (e < 0 || e >= num_experts)
      record_error(err_word, LM_DEVERR_BAD_EXPERT_ID);
    else
      s_active[e] = 1;
  }
  __syncwarp();
  int u = 0;
  for (int e = lane; e < num_experts; e += 32) u += s_active[e];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);

  if (u > num_slots) {
    // Working set above the slot count: the bank is not modified.
    for (int e = lane; e < num_experts; e += 32)
      if (s_active[e]) {
        const int s = expert_slot[e];
        group_src[e] = s >= 0 ? s : LM_SRC_HOST;
      }
    return;
  }
  const long long step = *step_counter;
  __syncwarp();
  if (lane == 0) *step_counter = step + 1;
  int hits = 0, misses = 0;  // counted by lane 0

  for (int base = 0; base < num_experts; base += 32) {
    unsigned act = __ballot_sync(0xffffffffu, base + lane < num_experts && s_active[base + lane]);
    while (act) {
      const int e = base + __ffs(act) - 1;
      act &= act - 1;
      int s = expert_slot[e];
      bool miss = false;
      if (s >= 0 && !s_loading[s]) {
        if (lane == 0) slot_last[s] = step;
      } else {
        miss = true;
        // first EMPTY slot
        s = -1;
        for (int b = 0; b < num_slots && s < 0; b += 32) {
          const int t = b + lane;
          const unsigned empty = __ballot_sync(0xffffffffu, t < num_slots && slot_owner[t] < 0);
          if (empty) s = b + __ffs(empty) - 1;
        }
        if (s < 0) {
          // READY slot (not loading in this call) with the least (last_used, slot id)
          long long best = 0x7fffffffffffffffll;
          int bi = 0x7fffffff;
          for (int t = lane; t < num_slots; t += 32) {
            if (s_loading[t]) continue;
            const long long lu = slot_last[t];
            if (lu < best || (lu == best && t < bi)) {
              best = lu;
              bi = t;
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const long long ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob < best || (ob == best && oi < bi)) {
              best = ob;
              bi = oi;
            }
          }
          s = bi < num_slots ? bi : -1;
        }
        if (s < 0) {  // cannot happen with u <= num_slots; keep the bank consistent
          if (lane == 0) record_error(err_word, LM_DEVERR_UNMAPPED_EXPERT);
          continue;
        }
        if (lane == 0) {
          const int old = slot_owner[s];
          if (old >= 0) expert_slot[old] = -1;
          slot_owner[s] = e;
          expert_slot[e] = s;
          slot_last[s] = step;
          s_loading[s] = 1;
        }
      }
      __syncwarp();
      if (lane == 0) {
        log2phy[e] = s;
        group_src[e] = miss ? (s | LM_SRC_MISS) : s;
        misses += miss ? 1 : 0;
        hits += miss ? 0 : 1;
      }
      __syncwarp();
    }
  }
  if (lane == 0 && hit_miss != nullptr) {
    hit_miss[0] += hits;
    hit_miss[1] += misses;
  }
}

}  // namespace
}  // namespace lm

using namespace lm;

extern "C" int lm_slot_plan(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                            int32_t num_slots, int32_t* slot_owner, int64_t* slot_last_used,
                            int32_t* expert_slot, int64_t* step_counter, int32_t* log2phy,
                            int32_t* group_src, int64_t* hit_miss_counts, int32_t* err_word,
                            void* stream) {
  if (num_pairs < 0 || num_experts <= 0 || num_experts > kPlanMaxExpertsSlots ||
      num_slots <= 0 || num_slots > kPlanMaxSlots)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_slot_plan: need 0 < num_experts <= 8192 and 0 < num_slots <= 1024");
  if ((num_pairs > 0 && topk_ids == nullptr) || slot_owner == nullptr ||
      slot_last_used == nullptr || expert_slot == nullptr || step_counter == nullptr ||
      log2phy == nullptr || group_src == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_slot_plan: null pointer");
  slot_plan_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, num_pairs, num_experts, num_slots, slot_owner,
      reinterpret_cast<long long*>(slot_last_used), expert_slot,
      reinterpret_cast<long long*>(step_counter), log2phy, group_src,
      reinterpret_cast<long long*>(hit_miss_counts), err_word);
  return launch_status("lm_slot_plan");
}
