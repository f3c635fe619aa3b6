// Routing-side kernels of the slot-bank MoE layer:
//   K1 router (scores -> grouped/plain top-k -> renorm -> scale -> bf16),
//   K2 expert histogram,
//   K4/K9 stable pair grouping (expert -> group/slot table, original pair order kept),
//   row gather (permute) and K8 weighted combine in the original top-k order.
// All kernels are deterministic: atomics only add integers.
#include <cfloat>
#include <cmath>
#include <mutex>
#include <string>

#include "lm_common.cuh"

namespace lm {
namespace {

constexpr int kRouteWarpsPerBlock = 8;
constexpr int kGroupTile = 512;  // pairs per tile in the grouping kernels
constexpr int kGroupTileWarps = kGroupTile / 32;
constexpr int kMaxGroups = 1024;

// Warp arg-max with ties broken toward the lower index. Returns the winner to all lanes.
__device__ __forceinline__ void warp_argmax(float& v, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
}

// Order-preserving image of a float key on uint32: a > b as floats <=> image(a) > image(b).
// -0.0 and +0.0 share an image (they compare equal as floats, so ties fall to the lower id),
// -inf maps above 0, and NaN maps to 0, below every key (a NaN key never wins a compare).
__device__ __forceinline__ uint32_t ordered_key(float f) {
  if (f != f) return 0u;
  uint32_t b = __float_as_uint(f);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Routes token t with one warp (expert e lives on lane e % 32, register slot e / 32): writes
// the token's top-k weights and ids and returns, on lane j < top_k, the j-th chosen expert.
template <int EPL>
__device__ __forceinline__ int route_one_token(const float* __restrict__ logits, int64_t t,
                                               int num_experts, int top_k, int scoring,
                                               int renorm, float scale,
                                               const float* __restrict__ bias, int n_group,
                                               int topk_group, uint16_t* __restrict__ w_bf16,
                                               float* __restrict__ w_f32,
                                               int32_t* __restrict__ ids, int lane,
                                               int num_shared = 0, int shared_base = 0) {
  const float* row = logits + t * num_experts;

  float lg[EPL], sc[EPL], key[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    lg[i] = (e < num_experts) ? __ldg(row + e) : -INFINITY;
  }

  if (scoring == LM_SCORING_SOFTMAX) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) m = fmaxf(m, lg[i]);
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      sc[i] = (e < num_experts) ? expf(lg[i] - m) : 0.f;
      s += sc[i];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < EPL; ++i) sc[i] *= inv;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) sc[i] = 1.0f / (1.0f + expf(-lg[i]));
  }

  // Selection key: the logit itself when no correction bias is given (scores are monotone
  // in the logit, so the chosen set and order are those of the scores, computed exactly);
  // otherwise score + bias as in group-limited routing with a correction bias.
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e >= num_experts) {
      key[i] = -INFINITY;
    } else if (bias != nullptr) {
      key[i] = sc[i] + __ldg(bias + e);
    } else {
      key[i] = lg[i];
    }
  }

  // Group-limited selection: keep the topk_group best groups (max key per group, or the sum
  // of the two best keys when a correction bias is used), ties toward the lower group id.
  if (n_group > 1 && topk_group < n_group) {  // n_group <= 32 (checked on the host)
    const int gsize = num_experts / n_group;
    unsigned keep_mask = 0;
    float gscore_mine = -INFINITY;  // lane g holds the score of group g
    for (int g = 0; g < n_group; ++g) {
      float b1 = -INFINITY;
      int i1 = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        if (e < num_experts && e / gsize == g && key[i] > b1) {
          b1 = key[i];
          i1 = e;
        }
      }
      float v = b1;
      int vi = i1;
      warp_argmax(v, vi);
      float score = v;
      if (bias != nullptr) {
        float b2 = -INFINITY;
        int i2 = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const int e = lane + 32 * i;
          if (e < num_experts && e / gsize == g && e != vi && key[i] > b2) {
            b2 = key[i];
            i2 = e;
          }
        }
        warp_argmax(b2, i2);
        score = v + (b2 == -INFINITY ? 0.f : b2);
      }
      if (lane == g) gscore_mine = score;
    }
    float gs = (lane < n_group) ? gscore_mine : -INFINITY;
    unsigned taken_groups = 0;
    for (int j = 0; j < topk_group; ++j) {
      float v = (lane < n_group && !((taken_groups >> lane) & 1u)) ? gs : -INFINITY;
      int vi = (lane < n_group && !((taken_groups >> lane) & 1u)) ? lane : 0x7fffffff;
      warp_argmax(v, vi);
      if (vi < 32) {
        keep_mask |= 1u << vi;
        taken_groups |= 1u << vi;
      }
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < num_experts && !((keep_mask >> (e / gsize)) & 1u)) key[i] = -INFINITY;
    }
  }

  // Top-k: k rounds of a warp arg-max over the unselected keys, on order-preserving integer
  // images of the keys so that each round is two warp reductions (max key, then the lowest
  // expert id holding it) instead of a shuffle tree.
  uint32_t okey[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) okey[i] = (lane + 32 * i < num_experts) ? ordered_key(key[i]) : 0u;
  float my_w = 0.f;
  int my_id = 0;
  unsigned taken = 0;
  for (int j = 0; j < top_k; ++j) {
    uint32_t best = 0;  // 0: no candidate (NaN keys map there and never win)
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      // experts of a lane ascend with i, so a strict compare keeps the lowest id of a tie
      if (!((taken >> i) & 1u) && okey[i] > best) {
        best = okey[i];
        bi = lane + 32 * i;
      }
    }
    const uint32_t top = __reduce_max_sync(0xffffffffu, best);
    int vi = static_cast<int>(
        __reduce_min_sync(0xffffffffu, (top != 0u && best == top) ? static_cast<uint32_t>(bi)
                                                                   : 0xffffffffu));
    if (top == 0u) vi = 0;  // only reachable with NaN logits: fall back to expert 0
    // Fetch the winner's score from its owner lane.
    const int owner = vi & 31;
    const int slot = vi >> 5;
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (i == slot) mine = sc[i];
    const float w = __shfl_sync(0xffffffffu, mine, owner);
    if (lane == owner) taken |= 1u << slot;
    if (lane == j) {
      my_w = w;
      my_id = vi;
    }
  }

  if (renorm) {
    const float s = warp_sum(lane < top_k ? my_w : 0.f);
    my_w = my_w / fmaxf(s, FLT_EPSILON);
  }
  my_w *= scale;
  // Rows hold the routed top-k followed by the fused shared suffix (num_shared > 0): ids
  // shared_base .. shared_base + num_shared - 1, each with weight 1.
  const int ld = top_k + num_shared;
  if (lane < top_k) {
    const int64_t o = t * ld + lane;
    w_bf16[o] = f32_to_bf16_bits(my_w);
    if (w_f32 != nullptr) w_f32[o] = my_w;
    ids[o] = my_id;
  } else if (lane < ld) {
    const int64_t o = t * ld + lane;
    w_bf16[o] = f32_to_bf16_bits(1.0f);
    if (w_f32 != nullptr) w_f32[o] = 1.0f;
    ids[o] = shared_base + (lane - top_k);
  }
  return my_id;
}

// One warp per token.
template <int EPL>
__global__ void __launch_bounds__(kRouteWarpsPerBlock * 32)
    route_topk_kernel(const float* __restrict__ logits, int64_t num_tokens, int num_experts,
                      int top_k, int scoring, int renorm, float scale,
                      const float* __restrict__ bias, int n_group, int topk_group,
                      uint16_t* __restrict__ w_bf16, float* __restrict__ w_f32,
                      int32_t* __restrict__ ids, int num_shared, int shared_base) {
  pdl_wait();
  pdl_trigger();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kRouteWarpsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= num_tokens) return;
  route_one_token<EPL>(logits, t, num_experts, top_k, scoring, renorm, scale, bias, n_group,
                       topk_group, w_bf16, w_f32, ids, lane, num_shared, shared_base);
}

__global__ void histogram_kernel(const int32_t* __restrict__ ids, int64_t num_pairs,
                                 int num_experts, int32_t* __restrict__ counts,
                                 int32_t* __restrict__ err_word) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int32_t s_hist[];
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) s_hist[e] = 0;
  __syncthreads();
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < num_pairs;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[p];
    if (e < 0 || e >= num_experts) {
      record_error(err_word, LM_DEVERR_BAD_EXPERT_ID);
      continue;
    }
    atomicAdd(&s_hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x)
    if (s_hist[e]) atomicAdd(&counts[e], s_hist[e]);
}

// Pairs / rows / tokens a call covers: the host bound, or fewer when the caller passes the
// count on the device (a count only known after earlier kernels, e.g. rows received).
__device__ __forceinline__ int64_t live_count(int64_t bound, const int32_t* count) {
  if (count == nullptr) return bound;
  const int64_t c = *count;
  return c < 0 ? 0 : (c < bound ? c : bound);
}

__device__ __forceinline__ int pair_group(const int32_t* ids, int64_t p, int64_t num_pairs,
                                          int num_experts, const int32_t* e2g, int num_groups,
                                          int32_t* err_word, bool report) {
  if (p >= num_pairs) return -2;
  const int e = ids[p];
  if (e < 0 || e >= num_experts) {
    if (report) record_error(err_word, LM_DEVERR_BAD_EXPERT_ID);
    return -1;
  }
  const int g = e2g[e];
  if (g < 0 || g >= num_groups) {
    if (report) record_error(err_word, LM_DEVERR_UNMAPPED_EXPERT);
    return -1;
  }
  return g;
}

// Pass 1: per-tile group counts.
__global__ void __launch_bounds__(kGroupTile)
    group_tile_count_kernel(const int32_t* __restrict__ ids, int64_t num_pairs, int num_experts,
                            const int32_t* __restrict__ e2g, int num_groups,
                            int32_t* __restrict__ tile_counts, int32_t* __restrict__ err_word,
                            const int32_t* __restrict__ count) {
  pdl_wait();
  pdl_trigger();
  num_pairs = live_count(num_pairs, count);
  extern __shared__ int32_t s_cnt[];
  for (int g = threadIdx.x; g < num_groups; g += blockDim.x) s_cnt[g] = 0;
  __syncthreads();
  const int64_t p = static_cast<int64_t>(blockIdx.x) * kGroupTile + threadIdx.x;
  const int g = pair_group(ids, p, num_pairs, num_experts, e2g, num_groups, err_word, true);
  if (g >= 0) atomicAdd(&s_cnt[g], 1);
  __syncthreads();
  int32_t* out = tile_counts + static_cast<int64_t>(blockIdx.x) * num_groups;
  for (int gg = threadIdx.x; gg < num_groups; gg += blockDim.x) out[gg] = s_cnt[gg];
}

// Pass 2 (one block): per-group exclusive scan over tiles, then exclusive scan over groups.
// The tiles of each group are split into chunks, one thread per (group, chunk), so that a
// thread has a short, independent run of loads: chunk sums, a scan over each group's
// chunks, then each thread rewrites its chunk as exclusive tile bases.
__global__ void __launch_bounds__(1024)
    group_scan_kernel(int32_t* __restrict__ tile_counts, int num_tiles, int num_groups,
                      int32_t* __restrict__ tile_base, int32_t* __restrict__ group_offsets) {
  pdl_wait();
  pdl_trigger();
  __shared__ int32_t s_tot[kMaxGroups];
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_part[1024];
  const int chunks = max(1, static_cast<int>(blockDim.x) / num_groups);
  const int chunk_len = (num_tiles + chunks - 1) / chunks;
  for (int i = threadIdx.x; i < chunks * num_groups; i += blockDim.x) {
    const int g = i % num_groups, c = i / num_groups;
    const int t0 = c * chunk_len, t1 = min(num_tiles, t0 + chunk_len);
    int sum = 0;
#pragma unroll 8
    for (int t = t0; t < t1; ++t) sum += tile_counts[static_cast<int64_t>(t) * num_groups + g];
    s_part[i] = sum;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < num_groups; g += blockDim.x) {
    int run = 0;
    for (int c = 0; c < chunks; ++c) {
      const int v = s_part[c * num_groups + g];
      s_part[c * num_groups + g] = run;
      run += v;
    }
    s_tot[g] = run;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < chunks * num_groups; i += blockDim.x) {
    const int g = i % num_groups, c = i / num_groups;
    const int t0 = c * chunk_len, t1 = min(num_tiles, t0 + chunk_len);
    int run = s_part[i];
#pragma unroll 8
    for (int t = t0; t < t1; ++t) {
      const int64_t o = static_cast<int64_t>(t) * num_groups + g;
      const int v = tile_counts[o];
      tile_base[o] = run;
      run += v;
    }
  }
  __syncthreads();
  // Exclusive scan of s_tot[0..num_groups) with one pass of 1024 threads.
  const int g = threadIdx.x;
  const int lane = g & 31, w = g >> 5;
  int v = (g < num_groups) ? s_tot[g] : 0;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int tt = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += tt;
  }
  if (lane == 31) s_warp[w] = incl;
  __syncthreads();
  if (w == 0) {
    int ws = s_warp[lane];
    int wi = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int tt = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += tt;
    }
    s_warp[lane] = wi - ws;  // exclusive warp prefix
  }
  __syncthreads();
  const int excl = s_warp[w] + incl - v;
  if (g < num_groups) group_offsets[g] = excl;
  if (g == num_groups - 1) group_offsets[num_groups] = excl + v;
}

// Pass 3: stable scatter. Rank inside the tile = pairs of the same group in earlier warps
// plus earlier lanes of this warp, so rows keep the original flat pair order.
__global__ void __launch_bounds__(kGroupTile)
    group_scatter_kernel(const int32_t* __restrict__ ids, int64_t num_pairs, int num_experts,
                         const int32_t* __restrict__ e2g, int num_groups,
                         const int32_t* __restrict__ tile_base,
                         const int32_t* __restrict__ group_offsets,
                         int32_t* __restrict__ pair_to_row, int32_t* __restrict__ row_to_pair,
                         const int32_t* __restrict__ count) {
  pdl_wait();
  pdl_trigger();
  num_pairs = live_count(num_pairs, count);
  extern __shared__ int32_t s_wcnt[];  // [kGroupTileWarps][num_groups]
  for (int i = threadIdx.x; i < kGroupTileWarps * num_groups; i += blockDim.x) s_wcnt[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * kGroupTile + threadIdx.x;
  const int g = pair_group(ids, p, num_pairs, num_experts, e2g, num_groups, nullptr, false);
  const unsigned peers = __match_any_sync(0xffffffffu, g);
  const unsigned lt = (1u << lane) - 1u;
  const int rank = __popc(peers & lt);
  if (g >= 0 && rank == 0) s_wcnt[w * num_groups + g] = __popc(peers);
  __syncthreads();
  if (g >= 0) {
    int off = rank;
    for (int ww = 0; ww < w; ++ww) off += s_wcnt[ww * num_groups + g];
    const int row =
        group_offsets[g] + tile_base[static_cast<int64_t>(blockIdx.x) * num_groups + g] + off;
    pair_to_row[p] = row;
    row_to_pair[row] = static_cast<int32_t>(p);
  } else if (g == -1) {
    pair_to_row[p] = -1;
  }
}

// All three passes for a call with at most kGroupTile pairs (decode), in one block of
// kGroupTile threads: per-warp group counts, the scan over groups, then the same stable
// scatter as the tiled passes, so the tables are identical to theirs without the scratch
// round trips between launches. sm: (1 + kGroupTileWarps) * num_groups int32 of shared
// memory; ids may be in global or shared memory.
__device__ __forceinline__ void group_one_tile(const int32_t* ids, int64_t num_pairs,
                                               int num_experts, const int32_t* __restrict__ e2g,
                                               int num_groups, int32_t* __restrict__ group_offsets,
                                               int32_t* __restrict__ pair_to_row,
                                               int32_t* __restrict__ row_to_pair,
                                               int32_t* __restrict__ err_word, int32_t* sm) {
  int32_t* s_base = sm;               // [num_groups]: first row of each group
  int32_t* s_wcnt = sm + num_groups;  // [kGroupTileWarps][num_groups]
  __shared__ int32_t s_warp[kGroupTileWarps];
  for (int i = threadIdx.x; i < kGroupTileWarps * num_groups; i += blockDim.x) s_wcnt[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int p = threadIdx.x;
  const int g = pair_group(ids, p, num_pairs, num_experts, e2g, num_groups, err_word, true);
  const unsigned peers = __match_any_sync(0xffffffffu, g);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (g >= 0 && rank == 0) s_wcnt[w * num_groups + g] = __popc(peers);
  __syncthreads();
  // thread t owns groups [t * gpt, t * gpt + gpt): totals, then a block exclusive scan
  const int gpt = (num_groups + kGroupTile - 1) / kGroupTile;
  const int ga = threadIdx.x * gpt;
  int mine = 0;
  for (int j = 0; j < gpt; ++j) {
    const int gg = ga + j;
    if (gg < num_groups)
      for (int ww = 0; ww < kGroupTileWarps; ++ww) mine += s_wcnt[ww * num_groups + gg];
  }
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp[w] = incl;
  __syncthreads();
  int before = 0;
  for (int ww = 0; ww < w; ++ww) before += s_warp[ww];
  int run = before + incl - mine;
  for (int j = 0; j < gpt; ++j) {
    const int gg = ga + j;
    if (gg < num_groups) {
      s_base[gg] = run;
      group_offsets[gg] = run;
      for (int ww = 0; ww < kGroupTileWarps; ++ww) run += s_wcnt[ww * num_groups + gg];
    }
  }
  if (ga < num_groups && ga + gpt >= num_groups) group_offsets[num_groups] = run;
  __syncthreads();
  if (g >= 0) {
    int row = s_base[g] + rank;
    for (int ww = 0; ww < w; ++ww) row += s_wcnt[ww * num_groups + g];
    pair_to_row[p] = row;
    row_to_pair[row] = p;
  } else if (g == -1) {
    pair_to_row[p] = -1;
  }
}

__global__ void __launch_bounds__(kGroupTile)
    group_single_tile_kernel(const int32_t* __restrict__ ids, int64_t num_pairs,
                             int num_experts, const int32_t* __restrict__ e2g, int num_groups,
                             int32_t* __restrict__ group_offsets,
                             int32_t* __restrict__ pair_to_row, int32_t* __restrict__ row_to_pair,
                             int32_t* __restrict__ err_word, const int32_t* __restrict__ count) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int32_t sm[];
  group_one_tile(ids, live_count(num_pairs, count), num_experts, e2g, num_groups, group_offsets,
                 pair_to_row, row_to_pair, err_word, sm);
}

// Router and grouping of a decode-sized call in one block (T * (top_k + num_shared) <=
// kGroupTile pairs): the warps route the tokens with the same device function as
// route_topk_kernel, the block synchronises (the ids it wrote are then visible to all its
// threads), and the pairs are grouped exactly as group_single_tile_kernel groups them. A
// layer whose experts are read in place groups by expert id, so its router can do both.
template <int EPL>
__global__ void __launch_bounds__(kGroupTile)
    route_group_kernel(const float* __restrict__ logits, int64_t num_tokens, int num_experts,
                       int top_k, int scoring, int renorm, float scale,
                       const float* __restrict__ bias, int n_group, int topk_group,
                       uint16_t* w_bf16, float* w_f32, int32_t* ids, int num_shared,
                       int num_experts_total, const int32_t* __restrict__ e2g, int num_groups,
                       int32_t* group_offsets, int32_t* pair_to_row, int32_t* row_to_pair,
                       int32_t* err_word) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int32_t sm[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t t = w; t < num_tokens; t += kGroupTileWarps)
    route_one_token<EPL>(logits, t, num_experts, top_k, scoring, renorm, scale, bias, n_group,
                         topk_group, w_bf16, w_f32, ids, lane, num_shared, num_experts);
  __syncthreads();
  group_one_tile(ids, num_tokens * (top_k + num_shared), num_experts_total, e2g, num_groups,
                 group_offsets, pair_to_row, row_to_pair, err_word, sm);
}

// Row gather through a second index: x_perm[r] = src[pair_src[row_to_pair[r]]], the source
// rows read at L2 (another GPU may have written them for this call; no stale L1 lines).
__global__ void permute_rows_gather_kernel(const uint16_t* __restrict__ src, int hidden_size,
                                           const int32_t* __restrict__ row_to_pair,
                                           const int32_t* __restrict__ pair_src,
                                           int64_t num_rows, uint16_t* __restrict__ x_perm,
                                           const int32_t* __restrict__ count) {
  pdl_wait();
  pdl_trigger();
  num_rows = live_count(num_rows, count);
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= num_rows) return;
  const int64_t row = pair_src[row_to_pair[r]];
  const uint4* in = reinterpret_cast<const uint4*>(src + row * hidden_size);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + r * hidden_size);
  for (int c = lane; c < hidden_size / 8; c += 32) dst[c] = __ldcg(in + c);
}

__global__ void permute_rows_kernel(const uint16_t* __restrict__ hidden, int hidden_size,
                                    const int32_t* __restrict__ row_to_pair, int top_k,
                                    int64_t num_rows, uint16_t* __restrict__ x_perm,
                                    const int32_t* __restrict__ count) {
  pdl_wait();
  pdl_trigger();
  num_rows = live_count(num_rows, count);
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= num_rows) return;
  const int64_t tok = row_to_pair[r] / top_k;
  const uint4* src = reinterpret_cast<const uint4*>(hidden + tok * hidden_size);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + r * hidden_size);
  for (int c = lane; c < hidden_size / 8; c += 32) dst[c] = __ldg(src + c);
}

__global__ void combine_kernel(const uint16_t* __restrict__ y_perm,
                               const int32_t* __restrict__ pair_to_row,
                               const uint16_t* __restrict__ w_bf16, int top_k, int hidden_size,
                               uint16_t* __restrict__ out, const int32_t* __restrict__ count) {
  __shared__ int32_t s_row[32];
  __shared__ float s_w[32];
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x;
  if (t >= live_count(gridDim.x, count)) return;
  if (threadIdx.x < top_k) {
    s_row[threadIdx.x] = pair_to_row[t * top_k + threadIdx.x];
    s_w[threadIdx.x] = bf16_bits_to_f32(w_bf16[t * top_k + threadIdx.x]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < hidden_size / 8; c += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    // up to 8 pairs' rows loaded at once, then accumulated in j order (the loads of a token's
    // rows are independent; only the sums are ordered)
    for (int j0 = 0; j0 < top_k; j0 += 8) {
      uint4 v[8];
      bool use[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int row = j0 + jj < top_k ? s_row[j0 + jj] : -1;
        use[jj] = row >= 0;
        if (use[jj])
          v[jj] = __ldg(
              reinterpret_cast<const uint4*>(y_perm + static_cast<int64_t>(row) * hidden_size) +
              c);
      }
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        if (!use[jj]) continue;
        const float w = s_w[j0 + jj];
        float a, b;
        unpack_bf16x2(v[jj].x, a, b);
        acc[0] += w * a;
        acc[1] += w * b;
        unpack_bf16x2(v[jj].y, a, b);
        acc[2] += w * a;
        acc[3] += w * b;
        unpack_bf16x2(v[jj].z, a, b);
        acc[4] += w * a;
        acc[5] += w * b;
        unpack_bf16x2(v[jj].w, a, b);
        acc[6] += w * a;
        acc[7] += w * b;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * hidden_size)[c] = o;
  }
}

}  // namespace
}  // namespace lm

using namespace lm;

namespace {
int check_route_args(int64_t num_tokens, int32_t num_experts, int32_t top_k,
                     int32_t scoring_func, int32_t num_expert_group, int32_t topk_group,
                     const float* logits, const uint16_t* topk_weights_bf16,
                     const int32_t* topk_ids) {
  if (num_tokens < 0 || num_experts <= 0 || num_experts > 256)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_route_topk: need 0 < num_experts <= 256");
  if (top_k <= 0 || top_k > 32 || top_k > num_experts)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_route_topk: need 0 < top_k <= min(32, E)");
  if (scoring_func != LM_SCORING_SOFTMAX && scoring_func != LM_SCORING_SIGMOID)
    return fail(LM_ERR_UNSUPPORTED, "lm_route_topk: scoring_func must be softmax or sigmoid");
  if (num_expert_group > 1) {
    if (num_expert_group > 32 || num_experts % num_expert_group != 0 || topk_group <= 0 ||
        topk_group > num_expert_group)
      return fail(LM_ERR_INVALID_ARGUMENT,
                  "lm_route_topk: grouped top-k needs n_group <= 32 dividing E and "
                  "0 < topk_group <= n_group");
    if (topk_group * (num_experts / num_expert_group) < top_k)
      return fail(LM_ERR_INVALID_ARGUMENT,
                  "lm_route_topk: topk_group groups hold fewer than top_k experts");
  }
  // an empty call may pass empty (null) tensors
  if (num_tokens > 0 &&
      (topk_weights_bf16 == nullptr || topk_ids == nullptr || logits == nullptr))
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_route_topk: null output or input pointer");
  return LM_OK;
}
}  // namespace

namespace {
int route_launch(const float* logits, int64_t num_tokens, int32_t num_experts, int32_t top_k,
                 int32_t scoring_func, int32_t renormalize, float routed_scaling_factor,
                 const float* e_score_correction_bias, int32_t num_expert_group,
                 int32_t topk_group, uint16_t* topk_weights_bf16, float* topk_weights_f32,
                 int32_t* topk_ids, int32_t num_shared, int32_t shared_base, void* stream,
                 const char* who) {
  if (num_tokens == 0) return LM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned blocks =
      static_cast<unsigned>((num_tokens + kRouteWarpsPerBlock - 1) / kRouteWarpsPerBlock);
  const int epl = (num_experts + 31) / 32;
  cudaError_t e = cudaSuccess;
#define LM_ROUTE_LAUNCH(N)                                                                   \
  e = launch_dependent(route_topk_kernel<N>, dim3(blocks), dim3(kRouteWarpsPerBlock * 32), 0, s, \
                       logits, num_tokens, num_experts, top_k, scoring_func, renormalize,    \
                       routed_scaling_factor, e_score_correction_bias, num_expert_group,     \
                       topk_group, topk_weights_bf16, topk_weights_f32, topk_ids, num_shared, \
                       shared_base)
  if (epl <= 1) {
    LM_ROUTE_LAUNCH(1);
  } else if (epl <= 2) {
    LM_ROUTE_LAUNCH(2);
  } else if (epl <= 4) {
    LM_ROUTE_LAUNCH(4);
  } else {
    LM_ROUTE_LAUNCH(8);
  }
#undef LM_ROUTE_LAUNCH
  if (e != cudaSuccess) return check_cuda(e, who);
  return launch_status(who);
}
}  // namespace

extern "C" int lm_route_topk(const float* logits, int64_t num_tokens, int32_t num_experts,
                             int32_t top_k, int32_t scoring_func, int32_t renormalize,
                             float routed_scaling_factor, const float* e_score_correction_bias,
                             int32_t num_expert_group, int32_t topk_group,
                             uint16_t* topk_weights_bf16, float* topk_weights_f32,
                             int32_t* topk_ids, void* stream) {
  int rc = check_route_args(num_tokens, num_experts, top_k, scoring_func, num_expert_group,
                            topk_group, logits, topk_weights_bf16, topk_ids);
  if (rc) return rc;
  return route_launch(logits, num_tokens, num_experts, top_k, scoring_func, renormalize,
                      routed_scaling_factor, e_score_correction_bias, num_expert_group,
                      topk_group, topk_weights_bf16, topk_weights_f32, topk_ids, 0, 0, stream,
                      "lm_route_topk");
}

extern "C" int lm_route_topk_shared(const float* logits, int64_t num_tokens,
                                    int32_t num_experts, int32_t top_k, int32_t scoring_func,
                                    int32_t renormalize, float routed_scaling_factor,
                                    const float* e_score_correction_bias,
                                    int32_t num_expert_group, int32_t topk_group,
                                    int32_t num_shared, uint16_t* topk_weights_bf16,
                                    float* topk_weights_f32, int32_t* topk_ids, void* stream) {
  int rc = check_route_args(num_tokens, num_experts, top_k, scoring_func, num_expert_group,
                            topk_group, logits, topk_weights_bf16, topk_ids);
  if (rc) return rc;
  if (num_shared < 0 || top_k + num_shared > 32)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_route_topk_shared: need 0 <= num_shared and top_k + num_shared <= 32");
  return route_launch(logits, num_tokens, num_experts, top_k, scoring_func, renormalize,
                      routed_scaling_factor, e_score_correction_bias, num_expert_group,
                      topk_group, topk_weights_bf16, topk_weights_f32, topk_ids, num_shared,
                      num_experts, stream, "lm_route_topk_shared");
}

extern "C" int lm_route_group_small(const float* logits, int64_t num_tokens,
                                    int32_t num_experts, int32_t top_k, int32_t scoring_func,
                                    int32_t renormalize, float routed_scaling_factor,
                                    const float* e_score_correction_bias,
                                    int32_t num_expert_group, int32_t topk_group,
                                    int32_t num_shared, uint16_t* topk_weights_bf16,
                                    float* topk_weights_f32, int32_t* topk_ids,
                                    int32_t num_experts_total, const int32_t* expert_to_group,
                                    int32_t num_groups, int32_t* group_offsets,
                                    int32_t* pair_to_row, int32_t* row_to_pair,
                                    int32_t* err_word, void* stream) {
  int rc = check_route_args(num_tokens, num_experts, top_k, scoring_func, num_expert_group,
                            topk_group, logits, topk_weights_bf16, topk_ids);
  if (rc) return rc;
  if (num_shared < 0 || top_k + num_shared > 32)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_route_group_small: need 0 <= num_shared and top_k + num_shared <= 32");
  const int64_t pairs = num_tokens * (top_k + num_shared);
  if (pairs <= 0 || pairs > kGroupTile)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_route_group_small: need 0 < num_tokens * (top_k + num_shared) <= 512");
  if (num_experts_total < num_experts + num_shared || num_groups <= 0 || num_groups > 16384 ||
      expert_to_group == nullptr || group_offsets == nullptr || pair_to_row == nullptr ||
      row_to_pair == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_route_group_small: bad grouping arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = sizeof(int32_t) * (1 + kGroupTileWarps) * num_groups;
  const int epl = (num_experts + 31) / 32;
  cudaError_t e = cudaSuccess;
#define LM_ROUTE_GROUP_LAUNCH(N)                                                               \
  do {                                                                                         \
    if (smem > 48 * 1024) {                                                                    \
      rc = check_cuda(cudaFuncSetAttribute(route_group_kernel<N>,                              \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                           static_cast<int>(smem)),                            \
                      "lm_route_group_small: smem attribute");                                \
      if (rc) return rc;                                                                       \
    }                                                                                          \
    e = launch_dependent(route_group_kernel<N>, dim3(1), dim3(kGroupTile), smem, s, logits,   \
                         num_tokens, num_experts, top_k, scoring_func, renormalize,            \
                         routed_scaling_factor, e_score_correction_bias, num_expert_group,     \
                         topk_group, topk_weights_bf16, topk_weights_f32, topk_ids,            \
                         num_shared, num_experts_total, expert_to_group, num_groups,           \
                         group_offsets, pair_to_row, row_to_pair, err_word);                   \
  } while (0)
  if (epl <= 1) {
    LM_ROUTE_GROUP_LAUNCH(1);
  } else if (epl <= 2) {
    LM_ROUTE_GROUP_LAUNCH(2);
  } else if (epl <= 4) {
    LM_ROUTE_GROUP_LAUNCH(4);
  } else {
    LM_ROUTE_GROUP_LAUNCH(8);
  }
#undef LM_ROUTE_GROUP_LAUNCH
  if (e != cudaSuccess) return check_cuda(e, "lm_route_group_small");
  return launch_status("lm_route_group_small");
}

extern "C" int lm_expert_histogram(const int32_t* topk_ids, int64_t num_pairs,
                                   int32_t num_experts, int32_t* counts, int32_t* err_word,
                                   void* stream) {
  if (num_pairs < 0 || num_experts <= 0 || num_experts > 16384 || counts == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_expert_histogram: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(counts, 0, sizeof(int32_t) * num_experts, s),
                      "lm_expert_histogram: memset");
  if (rc) return rc;
  if (num_pairs == 0) return LM_OK;
  const int threads = 256;
  int64_t blocks64 = (num_pairs + threads - 1) / threads;
  const unsigned blocks = static_cast<unsigned>(blocks64 > 1184 ? 1184 : blocks64);
  histogram_kernel<<<blocks, threads, sizeof(int32_t) * num_experts, s>>>(
      topk_ids, num_pairs, num_experts, counts, err_word);
  return launch_status("lm_expert_histogram");
}

extern "C" int64_t lm_build_groups_scratch_elems(int64_t num_pairs, int32_t num_groups) {
  if (num_pairs < 0 || num_groups <= 0) return 0;
  const int64_t tiles = (num_pairs + kGroupTile - 1) / kGroupTile;
  return 2 * (tiles > 0 ? tiles : 1) * static_cast<int64_t>(num_groups);
}

namespace {

// Grouping passes on caller-chosen scratch (2 * tiles * num_groups int32, fully written by
// the passes themselves, so it needs no clearing between calls).
int build_groups_impl(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                      const int32_t* expert_to_group, int32_t num_groups,
                      int32_t* group_offsets, int32_t* pair_to_row, int32_t* row_to_pair,
                      int32_t* scratch, int32_t* err_word, cudaStream_t s,
                      const int32_t* count = nullptr) {
  if (num_pairs > 0 && num_pairs <= kGroupTile) {
    const size_t smem = sizeof(int32_t) * (1 + kGroupTileWarps) * num_groups;
    if (smem > 48 * 1024) {
      int rc = check_cuda(cudaFuncSetAttribute(group_single_tile_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem)),
                          "lm_build_groups: smem attribute");
      if (rc) return rc;
    }
    const cudaError_t e =
        launch_dependent(group_single_tile_kernel, dim3(1), dim3(kGroupTile), smem, s, topk_ids,
                         num_pairs, num_experts, expert_to_group, num_groups, group_offsets,
                         pair_to_row, row_to_pair, err_word, count);
    if (e != cudaSuccess) return check_cuda(e, "lm_build_groups: single tile");
    return launch_status("lm_build_groups: single tile");
  }
  const int64_t tiles64 = (num_pairs + kGroupTile - 1) / kGroupTile;
  const int tiles = static_cast<int>(tiles64 > 0 ? tiles64 : 1);
  int32_t* tile_counts = scratch;
  int32_t* tile_base = scratch + static_cast<int64_t>(tiles) * num_groups;
  if (num_pairs == 0) {
    int rc = check_cuda(cudaMemsetAsync(tile_counts, 0, sizeof(int32_t) * num_groups, s),
                        "lm_build_groups: memset");
    if (rc) return rc;
  } else {
    const cudaError_t e = launch_dependent(
        group_tile_count_kernel, dim3(tiles), dim3(kGroupTile), sizeof(int32_t) * num_groups, s,
        topk_ids, num_pairs, num_experts, expert_to_group, num_groups, tile_counts, err_word,
        count);
    if (e != cudaSuccess) return check_cuda(e, "lm_build_groups: count");
    int rc = launch_status("lm_build_groups: count");
    if (rc) return rc;
  }
  const cudaError_t es = launch_dependent(group_scan_kernel, dim3(1), dim3(1024), 0, s,
                                          tile_counts, tiles, num_groups, tile_base,
                                          group_offsets);
  if (es != cudaSuccess) return check_cuda(es, "lm_build_groups: scan");
  int rc = launch_status("lm_build_groups: scan");
  if (rc || num_pairs == 0) return rc;
  const size_t smem = sizeof(int32_t) * kGroupTileWarps * num_groups;
  if (smem > 48 * 1024) {
    rc = check_cuda(cudaFuncSetAttribute(group_scatter_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)),
                    "lm_build_groups: smem attribute");
    if (rc) return rc;
  }
  const cudaError_t ec = launch_dependent(group_scatter_kernel, dim3(tiles), dim3(kGroupTile),
                                          smem, s, topk_ids, num_pairs, num_experts,
                                          expert_to_group, num_groups, tile_base, group_offsets,
                                          pair_to_row, row_to_pair, count);
  if (ec != cudaSuccess) return check_cuda(ec, "lm_build_groups: scatter");
  return launch_status("lm_build_groups: scatter");
}

int check_group_args(const char* who, const int32_t* topk_ids, int64_t num_pairs,
                     int32_t num_experts, const int32_t* expert_to_group, int32_t num_groups,
                     const int32_t* group_offsets, const int32_t* pair_to_row,
                     const int32_t* row_to_pair) {
  if (num_pairs < 0 || num_experts <= 0 || num_groups <= 0 || num_groups > kMaxGroups)
    return fail(LM_ERR_INVALID_ARGUMENT,
                std::string(who) + ": need num_pairs >= 0 and 0 < num_groups <= 1024");
  if (group_offsets == nullptr || expert_to_group == nullptr ||
      (num_pairs > 0 && (topk_ids == nullptr || pair_to_row == nullptr || row_to_pair == nullptr)))
    return fail(LM_ERR_INVALID_ARGUMENT, std::string(who) + ": null pointer");
  return LM_OK;
}

// Scratch of lm_build_groups_noalloc: one array per device that loads this library, kept
// until the process exits. Calls share it, so calls that overlap on the GPU race.
static __device__ __align__(256) int32_t g_group_scratch[LM_NOALLOC_GROUP_SCRATCH_ELEMS];

// Device address of g_group_scratch for the current device, resolved once per device with
// that device current (host code only sees a host-side shadow under the symbol's name).
int noalloc_scratch(int32_t** out) {
  static std::mutex mu;
  static int32_t* ptrs[64] = {nullptr};
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "lm_build_groups_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(LM_ERR_UNSUPPORTED, "lm_build_groups_noalloc: device index >= 64");
  std::lock_guard<std::mutex> lk(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_group_scratch),
                    "lm_build_groups_noalloc: cudaGetSymbolAddress");
    if (rc) return rc;
    ptrs[dev] = static_cast<int32_t*>(p);
  }
  *out = ptrs[dev];
  return LM_OK;
}

}  // namespace

extern "C" int lm_build_groups(const int32_t* topk_ids, int64_t num_pairs, int32_t num_experts,
                               const int32_t* expert_to_group, int32_t num_groups,
                               int32_t* group_offsets, int32_t* pair_to_row,
                               int32_t* row_to_pair, int32_t* scratch, int64_t scratch_elems,
                               int32_t* err_word, void* stream) {
  int rc = check_group_args("lm_build_groups", topk_ids, num_pairs, num_experts,
                            expert_to_group, num_groups, group_offsets, pair_to_row, row_to_pair);
  if (rc) return rc;
  const int64_t need = lm_build_groups_scratch_elems(num_pairs, num_groups);
  if (scratch == nullptr || scratch_elems < need)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_build_groups: scratch too small (need " + std::to_string(need) + " int32)");
  return build_groups_impl(topk_ids, num_pairs, num_experts, expert_to_group, num_groups,
                           group_offsets, pair_to_row, row_to_pair, scratch, err_word,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int lm_build_groups_count(const int32_t* topk_ids, int64_t max_pairs,
                                     const int32_t* num_pairs_dev, int32_t num_experts,
                                     const int32_t* expert_to_group, int32_t num_groups,
                                     int32_t* group_offsets, int32_t* pair_to_row,
                                     int32_t* row_to_pair, int32_t* scratch,
                                     int64_t scratch_elems, int32_t* err_word, void* stream) {
  if (num_pairs_dev == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_build_groups_count: null pair count");
  int rc = check_group_args("lm_build_groups_count", topk_ids, max_pairs, num_experts,
                            expert_to_group, num_groups, group_offsets, pair_to_row, row_to_pair);
  if (rc) return rc;
  const int64_t need = lm_build_groups_scratch_elems(max_pairs, num_groups);
  if (scratch == nullptr || scratch_elems < need)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_build_groups_count: scratch too small (need " + std::to_string(need) +
                    " int32)");
  return build_groups_impl(topk_ids, max_pairs, num_experts, expert_to_group, num_groups,
                           group_offsets, pair_to_row, row_to_pair, scratch, err_word,
                           static_cast<cudaStream_t>(stream), num_pairs_dev);
}

extern "C" int lm_build_groups_noalloc(const int32_t* topk_ids, int64_t num_pairs,
                                       int32_t num_experts, const int32_t* expert_to_group,
                                       int32_t num_groups, int32_t* group_offsets,
                                       int32_t* pair_to_row, int32_t* row_to_pair,
                                       int32_t* err_word, void* stream) {
  int rc = check_group_args("lm_build_groups_noalloc", topk_ids, num_pairs, num_experts,
                            expert_to_group, num_groups, group_offsets, pair_to_row, row_to_pair);
  if (rc) return rc;
  const int64_t need = lm_build_groups_scratch_elems(num_pairs, num_groups);
  if (need > LM_NOALLOC_GROUP_SCRATCH_ELEMS)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_build_groups_noalloc: num_pairs=" + std::to_string(num_pairs) +
                    " with num_groups=" + std::to_string(num_groups) + " needs " +
                    std::to_string(need) + " int32 of scratch; the built-in array holds " +
                    std::to_string(LM_NOALLOC_GROUP_SCRATCH_ELEMS) +
                    " (use lm_build_groups with caller-owned scratch)");
  int32_t* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return build_groups_impl(topk_ids, num_pairs, num_experts, expert_to_group, num_groups,
                           group_offsets, pair_to_row, row_to_pair, scratch, err_word,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int lm_permute_rows(const uint16_t* hidden, int32_t hidden_size,
                               const int32_t* row_to_pair, int32_t top_k, int64_t num_rows,
                               uint16_t* x_perm, void* stream) {
  if (hidden_size <= 0 || hidden_size % 8 != 0 || top_k <= 0 || num_rows < 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_permute_rows: need hidden_size % 8 == 0");
  if (num_rows == 0) return LM_OK;
  const int warps = 8;
  const unsigned blocks = static_cast<unsigned>((num_rows + warps - 1) / warps);
  const cudaError_t e = launch_dependent(
      permute_rows_kernel, dim3(blocks), dim3(warps * 32), 0, static_cast<cudaStream_t>(stream),
      hidden, hidden_size, row_to_pair, top_k, num_rows, x_perm,
      static_cast<const int32_t*>(nullptr));
  if (e != cudaSuccess) return check_cuda(e, "lm_permute_rows");
  return launch_status("lm_permute_rows");
}

extern "C" int lm_permute_rows_gather_count(const uint16_t* src, int32_t hidden_size,
                                            const int32_t* row_to_pair, const int32_t* pair_src,
                                            int64_t max_rows, const int32_t* num_rows_dev,
                                            uint16_t* x_perm, void* stream) {
  if (hidden_size <= 0 || hidden_size % 8 != 0 || max_rows < 0 || num_rows_dev == nullptr ||
      (max_rows > 0 && (src == nullptr || row_to_pair == nullptr || pair_src == nullptr ||
                        x_perm == nullptr)))
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_permute_rows_gather_count: need hidden_size % 8 == 0, tables and a count");
  if (max_rows == 0) return LM_OK;
  const int warps = 8;
  const unsigned blocks = static_cast<unsigned>((max_rows + warps - 1) / warps);
  const cudaError_t e = launch_dependent(
      permute_rows_gather_kernel, dim3(blocks), dim3(warps * 32), 0,
      static_cast<cudaStream_t>(stream), src, hidden_size, row_to_pair, pair_src, max_rows,
      x_perm, num_rows_dev);
  if (e != cudaSuccess) return check_cuda(e, "lm_permute_rows_gather_count");
  return launch_status("lm_permute_rows_gather_count");
}

extern "C" int lm_permute_rows_count(const uint16_t* hidden, int32_t hidden_size,
                                     const int32_t* row_to_pair, int32_t top_k,
                                     int64_t max_rows, const int32_t* num_rows_dev,
                                     uint16_t* x_perm, void* stream) {
  if (hidden_size <= 0 || hidden_size % 8 != 0 || top_k <= 0 || max_rows < 0 ||
      num_rows_dev == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_permute_rows_count: need hidden_size % 8 == 0 and a row count");
  if (max_rows == 0) return LM_OK;
  const int warps = 8;
  const unsigned blocks = static_cast<unsigned>((max_rows + warps - 1) / warps);
  const cudaError_t e = launch_dependent(
      permute_rows_kernel, dim3(blocks), dim3(warps * 32), 0, static_cast<cudaStream_t>(stream),
      hidden, hidden_size, row_to_pair, top_k, max_rows, x_perm, num_rows_dev);
  if (e != cudaSuccess) return check_cuda(e, "lm_permute_rows_count");
  return launch_status("lm_permute_rows_count");
}

extern "C" int lm_moe_combine(const uint16_t* y_perm, const int32_t* pair_to_row,
                              const uint16_t* topk_weights_bf16, int64_t num_tokens,
                              int32_t top_k, int32_t hidden_size, uint16_t* out, void* stream) {
  if (num_tokens < 0 || top_k <= 0 || top_k > 32 || hidden_size <= 0 || hidden_size % 8 != 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_combine: need 0 < top_k <= 32 and hidden_size % 8 == 0");
  if (num_tokens == 0) return LM_OK;
  if (num_tokens > 0x7fffffff) return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_combine: too many tokens");
  int threads = hidden_size / 8;
  if (threads > 512) threads = 512;
  if (threads < 32) threads = 32;
  const cudaError_t e = launch_dependent(
      combine_kernel, dim3(static_cast<unsigned>(num_tokens)), dim3(threads), 0,
      static_cast<cudaStream_t>(stream), y_perm, pair_to_row, topk_weights_bf16, top_k,
      hidden_size, out, static_cast<const int32_t*>(nullptr));
  if (e != cudaSuccess) return check_cuda(e, "lm_moe_combine");
  return launch_status("lm_moe_combine");
}

extern "C" int lm_moe_combine_count(const uint16_t* y_perm, const int32_t* pair_to_row,
                                    const uint16_t* topk_weights_bf16, int64_t max_tokens,
                                    const int32_t* num_tokens_dev, int32_t top_k,
                                    int32_t hidden_size, uint16_t* out, void* stream) {
  if (max_tokens < 0 || max_tokens > 0x7fffffff || top_k <= 0 || top_k > 32 ||
      hidden_size <= 0 || hidden_size % 8 != 0 || num_tokens_dev == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_combine_count: need 0 < top_k <= 32, hidden_size % 8 == 0 and a count");
  if (max_tokens == 0) return LM_OK;
  int threads = hidden_size / 8;
  if (threads > 512) threads = 512;
  if (threads < 32) threads = 32;
  const cudaError_t e = launch_dependent(
      combine_kernel, dim3(static_cast<unsigned>(max_tokens)), dim3(threads), 0,
      static_cast<cudaStream_t>(stream), y_perm, pair_to_row, topk_weights_bf16, top_k,
      hidden_size, out, num_tokens_dev);
  if (e != cudaSuccess) return check_cuda(e, "lm_moe_combine_count");
  return launch_status("lm_moe_combine_count");
}
