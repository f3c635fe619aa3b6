// Expert-parallel exchange over peer memory (NVLink / NVSwitch), one process per GPU.
//
// Every rank owns one "region" allocated with cudaMalloc and mapped into every other rank's
// address space through CUDA IPC. Layout (lm_ep_layout): arrival flags of the dispatch and of
// the outputs (one int64 per source rank), the per-source row counts, the owner's exclusive
// prefix of those counts, and a capacity-strided receive area (source s writes its rows at
// [s * cap, s * cap + count)), plus the owner's output rows in compacted order.
//
//   dispatch (source r):  store each token's hidden row once into every owner holding any of
//                         its experts (or, per pair, each pair's row), with each pair's
//                         owner-local expert id and receive-row index; the last block stores
//                         the counts and raises r's flag in every owner.
//   receive  (owner o):   wait for every source's flag (bounded), prefix the counts, then
//                         compact the rows for the local expert MLP, or list only the received
//                         pairs' receive rows (the MLP gathers from the receive area itself).
//   outputs  (owner o):   the MLP writes its rows locally (with a pair-row table the sources
//                         read), or stores each row straight into its source's output area
//                         through row pointers (lm_ep_output_row_ptrs).
//   signal   (owner o):   raise o's output flag in every source once its outputs are written.
//   combine  (source r):  wait for every owner's output flag (bounded), then per token read
//                         its pairs' output rows (from the owners' memory, or from its own
//                         area when the owners pushed them) and reduce them in fp32 in the
//                         original top-k order.
// Every kernel here is launched with programmatic dependent launch and waits for its
// predecessor in the stream (griddepcontrol.wait) before it touches memory.
// A source only re-dispatches after its combine read every owner's outputs (stream order),
// and an owner only compacts / overwrites after every source's next dispatch flag, so the
// areas need no other barrier. Flags carry the call's epoch (the same on every rank).
// No kernel waits on a kernel of its own GPU; waits are bounded and report
// LM_DEVERR_WAIT_TIMEOUT. No TMA and no multicast: plain peer loads and stores.
#include <cstring>

#include "lm_common.cuh"

namespace lm {
namespace {

constexpr int kLayoutFields = 12;
enum : int { F_FLAG_DISPATCH = 0, F_FLAG_OUT, F_COUNTS, F_PREFIX, F_WAIT_STATUS, F_EPOCH,
             F_RECV_IDS, F_RECV_ROWIDX, F_PAIR_ROW, F_RECV_ROWS, F_OUT_ROWS, F_TOTAL };

int64_t align256(int64_t v) { return (v + 255) & ~static_cast<int64_t>(255); }

void layout(int G, int cap, int H, int64_t* off) {
  int64_t o = 0;
  off[F_FLAG_DISPATCH] = o;
  o = align256(o + 8ll * G);
  off[F_FLAG_OUT] = o;
  o = align256(o + 8ll * G);
  off[F_COUNTS] = o;
  o = align256(o + 4ll * G);
  off[F_PREFIX] = o;
  o = align256(o + 4ll * (G + 1));
  off[F_WAIT_STATUS] = o;  // this rank's last output wait: 0 every owner answered, 1 timed out
  o = align256(o + 4);
  off[F_EPOCH] = o;  // the rank's call counter on the device (epoch argument 0 reads it)
  o = align256(o + 8);
  off[F_RECV_IDS] = o;
  o = align256(o + 4ll * G * cap);
  off[F_RECV_ROWIDX] = o;  // receive-area row of each received pair (rows may be shared)
  o = align256(o + 4ll * G * cap);
  off[F_PAIR_ROW] = o;  // owner: output row of its received pair d (read by the sources)
  o = align256(o + 4ll * G * cap);
  off[F_RECV_ROWS] = o;
  o = align256(o + 2ll * G * cap * H);
  off[F_OUT_ROWS] = o;  // + one spare row at G * cap that no one reads
  o = align256(o + 2ll * (static_cast<int64_t>(G) * cap + 1) * H);
  off[F_TOTAL] = o;
}

struct Layout {
  int64_t off[kLayoutFields];
};

template <typename T>
__device__ __forceinline__ T* field(void* region, const Layout& L, int f) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(region) + L.off[f]);
}

// The call's epoch: the argument, or, when it is 0, the counter in the rank's own region that
// lm_ep_advance_epoch raised earlier in the stream (so a captured step replays with a new
// epoch every time).
__device__ __forceinline__ long long call_epoch(long long epoch, void* own_region,
                                                const Layout& L) {
  return epoch > 0 ? epoch : *field<volatile long long>(own_region, L, F_EPOCH);
}

__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until flags[s] >= epoch for every s < G, by one full warp; the result is the
// same in every lane (false on time-out).
__device__ bool wait_flags(const long long* flags, int G, long long epoch, int32_t* err_word) {
  const long long t0 = clock64();
  bool ok = true;
  for (int s = threadIdx.x; s < G && ok; s += 32) {
    while (ld_acquire_sys(flags + s) < epoch) {
      if (clock64() - t0 > LM_SPIN_LIMIT_CYCLES) {
        record_error(err_word, LM_DEVERR_WAIT_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(256)
    ep_dispatch_kernel(const uint16_t* __restrict__ hidden, int64_t num_pairs, int top_k, int H,
                       const int32_t* __restrict__ ids, int per_rank,
                       const int32_t* __restrict__ pair_to_row,
                       const int32_t* __restrict__ send_offsets, int rank, int G,
                       void* const* __restrict__ peers, Layout L, int cap, long long epoch,
                       int32_t* __restrict__ done, int32_t* __restrict__ err_word) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  epoch = call_epoch(epoch, peers[rank], L);
  // one warp per pair
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       p < num_pairs; p += warps) {
    const int e = ids[p];
    const int o = e / per_rank;
    if (e < 0 || o >= G) {
      if (lane == 0) record_error(err_word, LM_DEVERR_BAD_EXPERT_ID);
      continue;
    }
    const int pos = pair_to_row[p] - send_offsets[o];
    if (pos < 0 || pos >= cap) {
      if (lane == 0) record_error(err_word, LM_DEVERR_BAD_GROUP);
      continue;
    }
    void* region = peers[o];
    const int64_t slot = static_cast<int64_t>(rank) * cap + pos;
    if (lane == 0) {
      field<int32_t>(region, L, F_RECV_IDS)[slot] = e - o * per_rank;
      field<int32_t>(region, L, F_RECV_ROWIDX)[slot] = static_cast<int32_t>(slot);
    }
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (p / top_k) * static_cast<int64_t>(H));
    uint4* dst = reinterpret_cast<uint4*>(field<uint16_t>(region, L, F_RECV_ROWS) + slot * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = __ldg(src + c);
  }
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  for (int o = threadIdx.x; o < G; o += blockDim.x)
    field<int32_t>(peers[o], L, F_COUNTS)[rank] = send_offsets[o + 1] - send_offsets[o];
  __threadfence_system();
  __syncthreads();
  for (int o = threadIdx.x; o < G; o += blockDim.x)
    st_release_sys(field<long long>(peers[o], L, F_FLAG_DISPATCH) + rank, epoch);
  if (threadIdx.x == 0) *done = 0;  // ready for the next call
}

// Token slots of a deduplicated dispatch: block o walks the tokens in order and numbers those
// with at least one pair owned by o (tok_slot[t * G + o], -1 otherwise); tok_count[o] = their
// number. A token's row then crosses to owner o once, whatever its number of pairs there.
__global__ void __launch_bounds__(1024)
    ep_token_slots_kernel(const int32_t* __restrict__ ids, int64_t num_tokens, int top_k,
                          int per_rank, int G, int32_t* __restrict__ tok_slot,
                          int32_t* __restrict__ tok_count) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int o = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < num_tokens; base += blockDim.x) {
    const int64_t t = base + threadIdx.x;
    int mine = 0;
    if (t < num_tokens) {
      for (int j = 0; j < top_k; ++j) {
        const int e = ids[t * top_k + j];
        if (e >= 0 && e / per_rank == o) mine = 1;
      }
    }
    // block exclusive scan of the flags
    const unsigned ball = __ballot_sync(0xffffffffu, mine);
    const int before_in_warp = __popc(ball & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[wid] = __popc(ball);
    __syncthreads();
    if (wid == 0) {
      int v = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      if (lane < nw) warp_sums[lane] = v;  // inclusive
    }
    __syncthreads();
    const int warp_base = wid ? warp_sums[wid - 1] : 0;
    if (t < num_tokens) tok_slot[t * G + o] = mine ? carry + warp_base + before_in_warp : -1;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sums[nw - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) tok_count[o] = carry;
}

// Deduplicated dispatch: warps over (token, owner) copy each needed token row once into the
// owner's receive area at [rank * tok_cap + token slot]; threads over pairs store each pair's
// owner-local id and receive-area row index. Same flags / counts protocol as
// ep_dispatch_kernel (counts are pairs per owner).
__global__ void __launch_bounds__(256)
    ep_dispatch_tokens_kernel(const uint16_t* __restrict__ hidden, int64_t num_tokens,
                              int top_k, int H, const int32_t* __restrict__ ids, int per_rank,
                              const int32_t* __restrict__ pair_to_row,
                              const int32_t* __restrict__ send_offsets,
                              const int32_t* __restrict__ tok_slot, int rank, int G,
                              void* const* __restrict__ peers, Layout L, int cap, int tok_cap,
                              long long epoch, int32_t* __restrict__ done,
                              int32_t* __restrict__ err_word) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  epoch = call_epoch(epoch, peers[rank], L);
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t w0 = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t num_pairs = num_tokens * top_k;
  for (int64_t q = w0; q < num_tokens * G; q += warps) {
    const int64_t t = q / G;
    const int o = static_cast<int>(q - t * G);
    const int ts = tok_slot[q];
    if (ts < 0) continue;
    if (ts >= tok_cap) {
      if (lane == 0) record_error(err_word, LM_DEVERR_BAD_GROUP);
      continue;
    }
    const int64_t row = static_cast<int64_t>(rank) * tok_cap + ts;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + t * static_cast<int64_t>(H));
    uint4* dst = reinterpret_cast<uint4*>(field<uint16_t>(peers[o], L, F_RECV_ROWS) + row * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = __ldg(src + c);
  }
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < num_pairs;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = ids[p];
    const int o = e / per_rank;
    if (e < 0 || o >= G) {
      record_error(err_word, LM_DEVERR_BAD_EXPERT_ID);
      continue;
    }
    const int pos = pair_to_row[p] - send_offsets[o];
    const int ts = tok_slot[(p / top_k) * G + o];
    if (pos < 0 || pos >= cap || ts < 0 || ts >= tok_cap) {
      record_error(err_word, LM_DEVERR_BAD_GROUP);
      continue;
    }
    const int64_t slot = static_cast<int64_t>(rank) * cap + pos;
    field<int32_t>(peers[o], L, F_RECV_IDS)[slot] = e - o * per_rank;
    field<int32_t>(peers[o], L, F_RECV_ROWIDX)[slot] = rank * tok_cap + ts;
  }
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  for (int o = threadIdx.x; o < G; o += blockDim.x)
    field<int32_t>(peers[o], L, F_COUNTS)[rank] = send_offsets[o + 1] - send_offsets[o];
  __threadfence_system();
  __syncthreads();
  for (int o = threadIdx.x; o < G; o += blockDim.x)
    st_release_sys(field<long long>(peers[o], L, F_FLAG_DISPATCH) + rank, epoch);
  if (threadIdx.x == 0) *done = 0;  // ready for the next call
}

__global__ void __launch_bounds__(32)
    ep_receive_wait_kernel(void* region, Layout L, int G, int cap, long long epoch,
                           int32_t* __restrict__ total_out, int32_t* __restrict__ err_word) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  epoch = call_epoch(epoch, region, L);
  int32_t* prefix = field<int32_t>(region, L, F_PREFIX);
  if (!wait_flags(field<long long>(region, L, F_FLAG_DISPATCH), G, epoch, err_word)) {
    if (threadIdx.x == 0) {
      for (int s = 0; s <= G; ++s) prefix[s] = 0;
      *total_out = 0;
    }
    return;
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const volatile int32_t* counts = field<int32_t>(region, L, F_COUNTS);
    int run = 0;
    for (int s = 0; s < G; ++s) {
      int c = counts[s];
      if (c < 0 || c > cap) {
        record_error(err_word, LM_DEVERR_BAD_GROUP);
        c = 0;
      }
      prefix[s] = run;
      run += c;
    }
    prefix[G] = run;
    *total_out = run;
  }
}

__global__ void __launch_bounds__(256)
    ep_compact_kernel(void* region, Layout L, int G, int cap, int H,
                      uint16_t* __restrict__ rows_out, int32_t* __restrict__ ids_out) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  const int32_t* prefix = field<int32_t>(region, L, F_PREFIX);
  const int32_t* recv_ids = field<int32_t>(region, L, F_RECV_IDS);
  const int32_t* recv_rowidx = field<int32_t>(region, L, F_RECV_ROWIDX);
  const uint16_t* recv_rows = field<uint16_t>(region, L, F_RECV_ROWS);
  int32_t* pair_row = field<int32_t>(region, L, F_PAIR_ROW);
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       q < static_cast<int64_t>(G) * cap; q += warps) {
    const int s = static_cast<int>(q / cap), i = static_cast<int>(q - static_cast<int64_t>(s) * cap);
    const int n = prefix[s + 1] - prefix[s];
    if (i >= n) continue;
    const int64_t d = prefix[s] + i;
    if (lane == 0) {
      ids_out[d] = __ldcg(recv_ids + q);
      pair_row[d] = static_cast<int32_t>(d);  // outputs land in received order
    }
    const int64_t srow = __ldcg(recv_rowidx + q);
    const uint4* src = reinterpret_cast<const uint4*>(recv_rows + srow * H);
    uint4* dst = reinterpret_cast<uint4*>(rows_out + d * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = __ldcg(src + c);
  }
}

// Index-only compaction: the received pairs' receive-area slots and owner-local ids in
// received order (no row copy; the owner's grouped MLP gathers its rows from the slots).
__global__ void __launch_bounds__(256)
    ep_index_kernel(void* region, Layout L, int G, int cap, int32_t* __restrict__ slot_out,
                    int32_t* __restrict__ ids_out) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  const int32_t* prefix = field<int32_t>(region, L, F_PREFIX);
  const int32_t* recv_ids = field<int32_t>(region, L, F_RECV_IDS);
  const int32_t* recv_rowidx = field<int32_t>(region, L, F_RECV_ROWIDX);
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       q < static_cast<int64_t>(G) * cap; q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(q / cap), i = static_cast<int>(q - static_cast<int64_t>(s) * cap);
    if (i >= prefix[s + 1] - prefix[s]) continue;
    const int64_t d = prefix[s] + i;
    slot_out[d] = __ldcg(recv_rowidx + q);
    ids_out[d] = __ldcg(recv_ids + q);
  }
}

// Output row pointers for an owner that pushes its MLP outputs to the sources: grouped row r
// holds received pair d = row_to_pair[r], which source s sent at position pos (d = prefix[s]
// + pos); its output goes to source s's region, row rank * cap + pos of the output area. A
// row whose pair is out of range points at this region's spare row instead (and is recorded).
__global__ void __launch_bounds__(256)
    ep_output_ptrs_kernel(void* region, void* const* __restrict__ peers, Layout L, int G,
                          int cap, int H, int rank, const int32_t* __restrict__ row_to_pair,
                          const int32_t* __restrict__ count_dev, int max_rows,
                          uint16_t** __restrict__ ptrs, int32_t* __restrict__ err_word) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  const int32_t* prefix = field<int32_t>(region, L, F_PREFIX);
  uint16_t* spare = field<uint16_t>(region, L, F_OUT_ROWS) + static_cast<int64_t>(G) * cap * H;
  int n = *count_dev;
  if (n > max_rows) n = max_rows;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
    const int d = row_to_pair[r];
    uint16_t* dst = spare;
    if (d >= 0 && d < prefix[G]) {
      int src = 0;
      while (src + 1 < G && prefix[src + 1] <= d) ++src;
      const int pos = d - prefix[src];
      if (pos < cap)
        dst = field<uint16_t>(peers[src], L, F_OUT_ROWS) +
              (static_cast<int64_t>(rank) * cap + pos) * H;
      else
        record_error(err_word, LM_DEVERR_BAD_GROUP);
    } else {
      record_error(err_word, LM_DEVERR_BAD_GROUP);
    }
    ptrs[r] = dst;
  }
}

// Per-step exchange figures kept on the device (one launch instead of several small ones):
// stats[0] += pairs received, stats[1] += pairs kept local, stats[2] += rows stored into
// other ranks by the dispatch (token rows when tok_count is given, else remote pairs),
// stats[3] += pairs routed by this rank.
__global__ void ep_stats_kernel(const int32_t* __restrict__ total,
                                const int32_t* __restrict__ send_offsets,
                                const int32_t* __restrict__ tok_count, int64_t num_pairs,
                                int rank, int G, long long* __restrict__ stats) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  if (threadIdx.x != 0) return;
  const long long local = send_offsets[rank + 1] - send_offsets[rank];
  long long stored = num_pairs - local;
  if (tok_count != nullptr) {
    stored = 0;
    for (int o = 0; o < G; ++o)
      if (o != rank) stored += tok_count[o];
  }
  stats[0] += *total;
  stats[1] += local;
  stats[2] += stored;
  stats[3] += num_pairs;
}

// One more call on this rank: raise the region's epoch counter (read by the exchange kernels
// of the call when they are given epoch 0).
__global__ void ep_advance_epoch_kernel(void* region, Layout L) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  if (threadIdx.x == 0) *field<long long>(region, L, F_EPOCH) += 1;
}

__global__ void ep_signal_kernel(void* const* __restrict__ peers, Layout L, int rank, int G,
                                 long long epoch) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  epoch = call_epoch(epoch, peers[rank], L);
  __threadfence_system();
  for (int o = threadIdx.x; o < G; o += blockDim.x)
    st_release_sys(field<long long>(peers[o], L, F_FLAG_OUT) + rank, epoch);
}

// Waits for every owner's output flag; the outcome goes to the region's wait-status word,
// which the combine reads so that a timed-out call never reads rows that may still change.
__global__ void __launch_bounds__(32)
    ep_wait_out_kernel(void* region, Layout L, int G, long long epoch, int32_t* err_word) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  epoch = call_epoch(epoch, region, L);
  const bool ok = wait_flags(field<long long>(region, L, F_FLAG_OUT), G, epoch, err_word);
  if (threadIdx.x == 0) *field<int32_t>(region, L, F_WAIT_STATUS) = ok ? 0 : 1;
}

// One block per token; the same accumulation order and arithmetic as combine_kernel.
// After a timed-out output wait (the local wait-status word) nothing is read from the owners
// and the token's row is written as zeros; a pair whose position lies outside [0, cap) is
// recorded as LM_DEVERR_BAD_GROUP and contributes nothing (the same rule as the dispatch).
__global__ void ep_combine_kernel(const int32_t* __restrict__ ids,
                                  const uint16_t* __restrict__ w_bf16, int top_k, int H,
                                  int per_rank, const int32_t* __restrict__ pair_to_row,
                                  const int32_t* __restrict__ send_offsets, int rank, int G,
                                  void* const* __restrict__ peers, const void* local_region,
                                  Layout L, int cap, uint16_t* __restrict__ out,
                                  int32_t* __restrict__ err_word, int pushed) {
  pdl_wait();  // launched early (programmatic dependent launch)
  pdl_trigger();
  __shared__ const uint16_t* s_src[32];
  __shared__ float s_w[32];
  const int64_t t = blockIdx.x;
  const bool waited = *field<const int32_t>(const_cast<void*>(local_region), L, F_WAIT_STATUS) == 0;
  if (threadIdx.x < top_k) {
    const int64_t p = t * top_k + threadIdx.x;
    const int e = ids[p];
    const int o = e / per_rank;
    const uint16_t* src = nullptr;
    if (e < 0 || o >= G) {
      record_error(err_word, LM_DEVERR_BAD_EXPERT_ID);
    } else if (waited) {
      const int pos = pair_to_row[p] - send_offsets[o];
      if (pos < 0 || pos >= cap) {
        record_error(err_word, LM_DEVERR_BAD_GROUP);
      } else if (pushed) {
        // the owner stored the output into this rank's own area, block o
        src = field<uint16_t>(const_cast<void*>(local_region), L, F_OUT_ROWS) +
              (static_cast<int64_t>(o) * cap + pos) * H;
      } else {
        const int32_t* prefix = field<int32_t>(peers[o], L, F_PREFIX);
        const int32_t* prow = field<int32_t>(peers[o], L, F_PAIR_ROW);
        const int64_t row = __ldcg(prow + __ldcg(prefix + rank) + pos);
        src = field<uint16_t>(peers[o], L, F_OUT_ROWS) + row * H;
      }
    }
    s_src[threadIdx.x] = src;
    s_w[threadIdx.x] = bf16_bits_to_f32(w_bf16[p]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < top_k; ++j) {
      const uint16_t* src = s_src[j];
      if (src == nullptr) continue;
      const float w = s_w[j];
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src) + c);
      float a, b;
      unpack_bf16x2(v.x, a, b);
      acc[0] += w * a;
      acc[1] += w * b;
      unpack_bf16x2(v.y, a, b);
      acc[2] += w * a;
      acc[3] += w * b;
      unpack_bf16x2(v.z, a, b);
      acc[4] += w * a;
      acc[5] += w * b;
      unpack_bf16x2(v.w, a, b);
      acc[6] += w * a;
      acc[7] += w * b;
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * H)[c] = o;
  }
}

Layout make_layout(int G, int cap, int H) {
  Layout L;
  layout(G, cap, H, L.off);
  return L;
}

int check_ep(const char* who, int G, int cap, int H) {
  if (G <= 0 || G > 64 || cap <= 0 || H <= 0 || H % 8 != 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                std::string(who) + ": need 0 < world <= 64, cap > 0, hidden % 8 == 0");
  return LM_OK;
}

}  // namespace
}  // namespace lm

using namespace lm;

extern "C" int64_t lm_ep_region_bytes(int32_t world, int32_t cap, int32_t hidden_size) {
  if (world <= 0 || cap <= 0 || hidden_size <= 0) return 0;
  int64_t off[kLayoutFields];
  layout(world, cap, hidden_size, off);
  return off[F_TOTAL];
}

extern "C" int lm_ep_region_alloc(int64_t bytes, void** region) {
  if (bytes <= 0 || region == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_region_alloc: bad size or null output");
  void* p = nullptr;
  int rc = check_cuda(cudaMalloc(&p, static_cast<size_t>(bytes)), "lm_ep_region_alloc: cudaMalloc");
  if (rc) return rc;
  rc = check_cuda(cudaMemset(p, 0, static_cast<size_t>(bytes)), "lm_ep_region_alloc: cudaMemset");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *region = p;
  return LM_OK;
}

extern "C" int lm_ep_region_free(void* region) {
  if (region == nullptr) return LM_OK;
  return check_cuda(cudaFree(region), "lm_ep_region_free");
}

extern "C" int lm_ipc_get_handle(const void* region, void* handle_out) {
  if (region == nullptr || handle_out == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(region)), "lm_ipc_get_handle");
  if (rc) return rc;
  std::memcpy(handle_out, &h, sizeof(h));
  return LM_OK;
}

extern "C" int lm_ipc_open_handle(const void* handle, void** region_out) {
  if (handle == nullptr || region_out == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(region_out, h, cudaIpcMemLazyEnablePeerAccess),
                    "lm_ipc_open_handle");
}

extern "C" int lm_ipc_close_handle(void* region) {
  if (region == nullptr) return LM_OK;
  return check_cuda(cudaIpcCloseMemHandle(region), "lm_ipc_close_handle");
}

extern "C" int lm_ep_dispatch(const uint16_t* hidden, int64_t num_tokens, int32_t top_k,
                              int32_t hidden_size, const int32_t* topk_ids,
                              int32_t experts_per_rank, const int32_t* pair_to_row,
                              const int32_t* send_offsets, int32_t rank, int32_t world,
                              void* const* peer_regions, int32_t cap, int64_t epoch,
                              int32_t* done_counter, int32_t* err_word, void* stream) {
  int rc = check_ep("lm_ep_dispatch", world, cap, hidden_size);
  if (rc) return rc;
  if (num_tokens < 0 || top_k <= 0 || experts_per_rank <= 0 || rank < 0 || rank >= world ||
      epoch < 0 || done_counter == nullptr || peer_regions == nullptr ||
      send_offsets == nullptr || (num_tokens > 0 && (hidden == nullptr || topk_ids == nullptr ||
                                                     pair_to_row == nullptr)))
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_dispatch: bad arguments");
  if (num_tokens * top_k > cap)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_ep_dispatch: num_tokens * top_k exceeds the exchange capacity cap");
  if (reinterpret_cast<uintptr_t>(hidden) & 15)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_dispatch: hidden must be 16-byte aligned");
  const int64_t pairs = num_tokens * top_k;
  int64_t blocks = (pairs + 7) / 8;
  if (blocks < 1) blocks = 1;
  if (blocks > 1184) blocks = 1184;
  {
    const cudaError_t le_ = launch_dependent(ep_dispatch_kernel,
        dim3(static_cast<unsigned>(blocks)), dim3(256), 0, static_cast<cudaStream_t>(stream),
        hidden, pairs, top_k, hidden_size, topk_ids, experts_per_rank, pair_to_row, send_offsets,
        rank, world, peer_regions, make_layout(world, cap, hidden_size), cap, epoch, done_counter,
        err_word);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_dispatch_kernel");
  }
  return launch_status("lm_ep_dispatch");
}

extern "C" int lm_ep_dispatch_tokens(const uint16_t* hidden, int64_t num_tokens, int32_t top_k,
                                     int32_t hidden_size, const int32_t* topk_ids,
                                     int32_t experts_per_rank, const int32_t* pair_to_row,
                                     const int32_t* send_offsets, int32_t rank, int32_t world,
                                     void* const* peer_regions, int32_t cap, int64_t epoch,
                                     int32_t* tok_slot, int32_t* tok_count,
                                     int32_t* done_counter, int32_t* err_word, void* stream) {
  int rc = check_ep("lm_ep_dispatch_tokens", world, cap, hidden_size);
  if (rc) return rc;
  if (num_tokens < 0 || top_k <= 0 || experts_per_rank <= 0 || rank < 0 || rank >= world ||
      epoch < 0 || done_counter == nullptr || peer_regions == nullptr ||
      send_offsets == nullptr || tok_count == nullptr ||
      (num_tokens > 0 && (hidden == nullptr || topk_ids == nullptr || pair_to_row == nullptr ||
                          tok_slot == nullptr)))
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_dispatch_tokens: bad arguments");
  if (num_tokens * top_k > cap)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_ep_dispatch_tokens: num_tokens * top_k exceeds the exchange capacity cap");
  if (reinterpret_cast<uintptr_t>(hidden) & 15)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_dispatch_tokens: hidden must be 16-byte aligned");
  // a source's token rows start at rank * tok_cap inside the world * cap receive rows
  const int tok_cap = cap / top_k;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const cudaError_t le_ = launch_dependent(ep_token_slots_kernel, dim3(world), dim3(1024), 0, s,
        topk_ids, num_tokens, top_k, experts_per_rank, world, tok_slot, tok_count);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_token_slots_kernel");
  }
  rc = launch_status("lm_ep_dispatch_tokens: token slots");
  if (rc) return rc;
  int64_t blocks = (num_tokens * world + 7) / 8;
  if (blocks < 1) blocks = 1;
  if (blocks > 1184) blocks = 1184;
  {
    const cudaError_t le_ = launch_dependent(ep_dispatch_tokens_kernel,
        dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, hidden, num_tokens, top_k,
        hidden_size, topk_ids, experts_per_rank, pair_to_row, send_offsets, tok_slot, rank, world,
        peer_regions, make_layout(world, cap, hidden_size), cap, tok_cap, epoch, done_counter,
        err_word);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_dispatch_tokens_kernel");
  }
  return launch_status("lm_ep_dispatch_tokens");
}

extern "C" int lm_ep_receive(void* region, int32_t world, int32_t cap, int32_t hidden_size,
                             int64_t epoch, uint16_t* rows_out, int32_t* ids_out,
                             int32_t* total_out, int32_t* err_word, void* stream) {
  int rc = check_ep("lm_ep_receive", world, cap, hidden_size);
  if (rc) return rc;
  if (region == nullptr || rows_out == nullptr || ids_out == nullptr || total_out == nullptr ||
      epoch < 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_receive: bad arguments");
  const Layout L = make_layout(world, cap, hidden_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const cudaError_t le_ = launch_dependent(ep_receive_wait_kernel, dim3(1), dim3(32), 0, s,
        region, L, world, cap, epoch, total_out, err_word);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_receive_wait_kernel");
  }
  rc = launch_status("lm_ep_receive: wait");
  if (rc) return rc;
  int64_t blocks = (static_cast<int64_t>(world) * cap + 7) / 8;
  if (blocks > 1184) blocks = 1184;
  {
    const cudaError_t le_ = launch_dependent(ep_compact_kernel,
        dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, region, L, world, cap, hidden_size,
        rows_out, ids_out);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_compact_kernel");
  }
  return launch_status("lm_ep_receive: compact");
}

extern "C" int lm_ep_receive_index(void* region, int32_t world, int32_t cap,
                                   int32_t hidden_size, int64_t epoch, int32_t* slot_out,
                                   int32_t* ids_out, int32_t* total_out, int32_t* err_word,
                                   void* stream) {
  int rc = check_ep("lm_ep_receive_index", world, cap, hidden_size);
  if (rc) return rc;
  if (region == nullptr || slot_out == nullptr || ids_out == nullptr || total_out == nullptr ||
      epoch < 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_receive_index: bad arguments");
  const Layout L = make_layout(world, cap, hidden_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const cudaError_t le_ = launch_dependent(ep_receive_wait_kernel, dim3(1), dim3(32), 0, s,
        region, L, world, cap, epoch, total_out, err_word);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_receive_wait_kernel");
  }
  rc = launch_status("lm_ep_receive_index: wait");
  if (rc) return rc;
  int64_t blocks = (static_cast<int64_t>(world) * cap + 255) / 256;
  if (blocks > 1184) blocks = 1184;
  {
    const cudaError_t le_ = launch_dependent(ep_index_kernel, dim3(static_cast<unsigned>(blocks)),
        dim3(256), 0, s, region, L, world, cap, slot_out, ids_out);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_index_kernel");
  }
  return launch_status("lm_ep_receive_index: index");
}

extern "C" int64_t lm_ep_recv_rows_offset(int32_t world, int32_t cap, int32_t hidden_size) {
  if (world <= 0 || cap <= 0 || hidden_size <= 0) return -1;
  int64_t off[kLayoutFields];
  layout(world, cap, hidden_size, off);
  return off[F_RECV_ROWS];
}

extern "C" int64_t lm_ep_pair_rows_offset(int32_t world, int32_t cap, int32_t hidden_size) {
  if (world <= 0 || cap <= 0 || hidden_size <= 0) return -1;
  int64_t off[kLayoutFields];
  layout(world, cap, hidden_size, off);
  return off[F_PAIR_ROW];
}

extern "C" int64_t lm_ep_out_rows_offset(int32_t world, int32_t cap, int32_t hidden_size) {
  if (world <= 0 || cap <= 0 || hidden_size <= 0) return -1;
  int64_t off[kLayoutFields];
  layout(world, cap, hidden_size, off);
  return off[F_OUT_ROWS];
}

extern "C" int lm_ep_signal_outputs(void* const* peer_regions, int32_t rank, int32_t world,
                                    int32_t cap, int32_t hidden_size, int64_t epoch,
                                    void* stream) {
  int rc = check_ep("lm_ep_signal_outputs", world, cap, hidden_size);
  if (rc) return rc;
  if (peer_regions == nullptr || rank < 0 || rank >= world || epoch < 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_signal_outputs: bad arguments");
  {
    const cudaError_t le_ = launch_dependent(ep_signal_kernel, dim3(1), dim3(32), 0,
        static_cast<cudaStream_t>(stream), peer_regions, make_layout(world, cap, hidden_size),
        rank, world, epoch);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_signal_kernel");
  }
  return launch_status("lm_ep_signal_outputs");
}

namespace {
int combine_impl(const int32_t* topk_ids, const uint16_t* topk_weights_bf16, int64_t num_tokens,
                 int32_t top_k, int32_t hidden_size, int32_t experts_per_rank,
                 const int32_t* pair_to_row, const int32_t* send_offsets, int32_t rank,
                 int32_t world, void* const* peer_regions, void* local_region, int32_t cap,
                 int64_t epoch, uint16_t* out, int32_t* err_word, void* stream, int pushed) {
  int rc = check_ep("lm_ep_combine", world, cap, hidden_size);
  if (rc) return rc;
  if (top_k <= 0 || top_k > 32 || num_tokens < 0 || experts_per_rank <= 0 || rank < 0 ||
      rank >= world || epoch < 0 || peer_regions == nullptr || local_region == nullptr ||
      (num_tokens > 0 && (topk_ids == nullptr || topk_weights_bf16 == nullptr ||
                          pair_to_row == nullptr || send_offsets == nullptr || out == nullptr)))
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_combine: bad arguments");
  if (num_tokens * top_k > cap)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_ep_combine: num_tokens * top_k exceeds the exchange capacity cap");
  if (reinterpret_cast<uintptr_t>(out) & 15)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_combine: out must be 16-byte aligned");
  const Layout L = make_layout(world, cap, hidden_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const cudaError_t le_ = launch_dependent(ep_wait_out_kernel, dim3(1), dim3(32), 0, s,
        local_region, L, world, epoch, err_word);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_wait_out_kernel");
  }
  rc = launch_status("lm_ep_combine: wait");
  if (rc || num_tokens == 0) return rc;
  int threads = hidden_size / 8;
  if (threads > 256) threads = 256;
  if (threads < 32) threads = 32;
  {
    const cudaError_t le_ = launch_dependent(ep_combine_kernel,
        dim3(static_cast<unsigned>(num_tokens)), dim3(threads), 0, s, topk_ids, topk_weights_bf16,
        top_k, hidden_size, experts_per_rank, pair_to_row, send_offsets, rank, world, peer_regions,
        local_region, L, cap, out, err_word, pushed);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_combine_kernel");
  }
  return launch_status("lm_ep_combine");
}
}  // namespace

extern "C" int lm_ep_combine(const int32_t* topk_ids, const uint16_t* topk_weights_bf16,
                             int64_t num_tokens, int32_t top_k, int32_t hidden_size,
                             int32_t experts_per_rank, const int32_t* pair_to_row,
                             const int32_t* send_offsets, int32_t rank, int32_t world,
                             void* const* peer_regions, void* local_region, int32_t cap,
                             int64_t epoch, uint16_t* out, int32_t* err_word, void* stream) {
  return combine_impl(topk_ids, topk_weights_bf16, num_tokens, top_k, hidden_size,
                      experts_per_rank, pair_to_row, send_offsets, rank, world, peer_regions,
                      local_region, cap, epoch, out, err_word, stream, 0);
}

extern "C" int lm_ep_combine_local(const int32_t* topk_ids, const uint16_t* topk_weights_bf16,
                                   int64_t num_tokens, int32_t top_k, int32_t hidden_size,
                                   int32_t experts_per_rank, const int32_t* pair_to_row,
                                   const int32_t* send_offsets, int32_t rank, int32_t world,
                                   void* const* peer_regions, void* local_region, int32_t cap,
                                   int64_t epoch, uint16_t* out, int32_t* err_word,
                                   void* stream) {
  return combine_impl(topk_ids, topk_weights_bf16, num_tokens, top_k, hidden_size,
                      experts_per_rank, pair_to_row, send_offsets, rank, world, peer_regions,
                      local_region, cap, epoch, out, err_word, stream, 1);
}

extern "C" int lm_ep_advance_epoch(void* region, int32_t world, int32_t cap,
                                   int32_t hidden_size, void* stream) {
  int rc = check_ep("lm_ep_advance_epoch", world, cap, hidden_size);
  if (rc) return rc;
  if (region == nullptr) return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_advance_epoch: null region");
  const cudaError_t le_ = launch_dependent(ep_advance_epoch_kernel, dim3(1), dim3(32), 0,
                                           static_cast<cudaStream_t>(stream), region,
                                           make_layout(world, cap, hidden_size));
  if (le_ != cudaSuccess) return check_cuda(le_, "ep_advance_epoch_kernel");
  return launch_status("lm_ep_advance_epoch");
}

extern "C" int lm_ep_step_stats(const int32_t* total, const int32_t* send_offsets,
                                const int32_t* tok_count, int64_t num_pairs, int32_t rank,
                                int32_t world, int64_t* stats, void* stream) {
  if (total == nullptr || send_offsets == nullptr || stats == nullptr || rank < 0 ||
      rank >= world || num_pairs < 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_step_stats: bad arguments");
  {
    const cudaError_t le_ = launch_dependent(ep_stats_kernel, dim3(1), dim3(32), 0,
        static_cast<cudaStream_t>(stream), total, send_offsets, tok_count, num_pairs, rank, world,
        reinterpret_cast<long long*>(stats));
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_stats_kernel");
  }
  return launch_status("lm_ep_step_stats");
}

extern "C" int lm_ep_output_row_ptrs(void* region, int32_t world, int32_t cap,
                                     int32_t hidden_size, int32_t rank,
                                     void* const* peer_regions, const int32_t* row_to_pair,
                                     const int32_t* count_dev, int32_t max_rows,
                                     uint16_t** row_ptrs_out, int32_t* err_word, void* stream) {
  int rc = check_ep("lm_ep_output_row_ptrs", world, cap, hidden_size);
  if (rc) return rc;
  if (region == nullptr || peer_regions == nullptr || rank < 0 || rank >= world ||
      max_rows < 0 || (max_rows > 0 && (row_to_pair == nullptr || count_dev == nullptr ||
                                        row_ptrs_out == nullptr)))
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_ep_output_row_ptrs: bad arguments");
  if (max_rows == 0) return LM_OK;
  int blocks = (max_rows + 255) / 256;
  if (blocks > 1184) blocks = 1184;
  {
    const cudaError_t le_ = launch_dependent(ep_output_ptrs_kernel, dim3(blocks), dim3(256), 0,
        static_cast<cudaStream_t>(stream), region, peer_regions,
        make_layout(world, cap, hidden_size), world, cap, hidden_size, rank, row_to_pair,
        count_dev, max_rows, row_ptrs_out, err_word);
    if (le_ != cudaSuccess) return check_cuda(le_, "ep_output_ptrs_kernel");
  }
  return launch_status("lm_ep_output_row_ptrs");
}
