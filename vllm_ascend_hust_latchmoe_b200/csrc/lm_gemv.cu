// Decode path of the grouped expert MLP: small groups (a few tokens per expert), so the
// layer is bound by streaming each active expert's weights from HBM exactly once.
//
// Each warp owns 16 weight rows and streams them with 128-bit loads (4 lanes cover the 64
// contiguous bytes of one row per 32-element K block). The tokens of the group sit on the
// N side of an m16n8k16 MMA, so one weight load serves up to 8 tokens per MMA and all token
// chunks of the group while it is in registers. The reduction over K is order-free, so a
// lane's 8 consecutive K elements are mapped onto the MMA fragment's K positions with a
// fixed permutation applied identically to the weights and the tokens.
//
// gate_up: warp rows = 8 gate rows (j0..j0+7) + the 8 matching up rows, so each lane ends up
// holding gate and up for the same (token, j) and applies SiLU(gate) * up in registers.
// down: warp rows = 16 consecutive output columns of the hidden dimension.
// Weights are in the tile-contiguous bank layout [N/128][K/64][128][64]: a row's 64-element
// K chunk is 128 contiguous bytes and the 8 rows a load instruction touches share a tile.
#include <cstdio>
#include <mutex>
#include <utility>
#include <vector>

#include "lm_common.cuh"
#include "lm_tmap.cuh"

namespace lm {
namespace {

constexpr int kGemvWarps = 8;

__device__ __forceinline__ uint4 ld_stream_16(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Plain 16-byte load, for weights read from the pinned host store over PCIe.
__device__ __forceinline__ uint4 ld_sys_16(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_16(uint16_t* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Weight source of one warp in the offload variant: loads from `sys` memory (the host store)
// use plain loads; when `c_lo`/`c_hi` are set every loaded chunk is also stored there (the
// expert's slot), so a missed expert crosses PCIe once and is cached for later calls.
struct WeightSrc {
  bool sys;
  uint16_t* c_lo;
  uint16_t* c_hi;
};

__device__ __forceinline__ uint4 ld_weight(const uint16_t* p, const WeightSrc& src) {
  return src.sys ? ld_sys_16(p) : ld_stream_16(p);
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Element offset of (row, 0) of a [N, K] matrix in the tile-contiguous layout.
__device__ __forceinline__ int64_t tiled_row_base(int row, int K) {
  return (static_cast<int64_t>(row >> 7) * (K >> 6)) * 8192 + (row & 127) * 64;
}

// Offset of the 32-element K block `kb` from a row base in the tile-contiguous layout.
__device__ __forceinline__ int tiled_kblock(int kb) { return (kb >> 1) * 8192 + (kb & 1) * 32; }

// acc[n] += W[16 rows, klen] x X[8 tokens of chunk n, klen]^T for one warp.
// w_lo: tiled row base of this lane's fragment row 0..7 (row = lane/4), w_hi: rows 8..15.
// xrow[n]: this lane's token row for chunk n (token = chunk*8 + lane/4), or nullptr.
template <int NC, bool OFFLOAD = false>
__device__ __forceinline__ void warp_tile(const uint16_t* __restrict__ w_lo,
                                          const uint16_t* __restrict__ w_hi,
                                          const uint16_t* const (&xrow)[NC], int klen,
                                          float (&acc)[NC][4], const WeightSrc& src = {}) {
  const int c8 = (threadIdx.x & 3) * 8;
  const int nblk = klen / 32;
  constexpr int U = 4;
  int kb = 0;
  for (; kb + U <= nblk; kb += U) {
    uint4 wl[U], wh[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int o = tiled_kblock(kb + u) + c8;
      if constexpr (OFFLOAD) {
        wl[u] = ld_weight(w_lo + o, src);
        wh[u] = ld_weight(w_hi + o, src);
      } else {
        wl[u] = ld_stream_16(w_lo + o);
        wh[u] = ld_stream_16(w_hi + o);
      }
    }
    if constexpr (OFFLOAD) {
      if (src.c_lo != nullptr) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int o = tiled_kblock(kb + u) + c8;
          st_16(src.c_lo + o, wl[u]);
          st_16(src.c_hi + o, wh[u]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        uint4 x = make_uint4(0, 0, 0, 0);
        if (xrow[n] != nullptr) x = __ldg(reinterpret_cast<const uint4*>(xrow[n] + (kb + u) * 32 + c8));
        mma_16816(acc[n], wl[u].x, wh[u].x, wl[u].y, wh[u].y, x.x, x.y);
        mma_16816(acc[n], wl[u].z, wh[u].z, wl[u].w, wh[u].w, x.z, x.w);
      }
    }
  }
  for (; kb < nblk; ++kb) {
    const int o = tiled_kblock(kb) + c8;
    uint4 wl, wh;
    if constexpr (OFFLOAD) {
      wl = ld_weight(w_lo + o, src);
      wh = ld_weight(w_hi + o, src);
      if (src.c_lo != nullptr) {
        st_16(src.c_lo + o, wl);
        st_16(src.c_hi + o, wh);
      }
    } else {
      wl = ld_stream_16(w_lo + o);
      wh = ld_stream_16(w_hi + o);
    }
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      uint4 x = make_uint4(0, 0, 0, 0);
      if (xrow[n] != nullptr) x = __ldg(reinterpret_cast<const uint4*>(xrow[n] + kb * 32 + c8));
      mma_16816(acc[n], wl.x, wh.x, wl.y, wh.y, x.x, x.y);
      mma_16816(acc[n], wl.z, wh.z, wl.w, wh.w, x.z, x.w);
    }
  }
}

__device__ __forceinline__ bool load_group(const int32_t* group_offsets,
                                           const int32_t* group_bank_row, int g,
                                           int64_t bank_rows, int32_t* err_word, int& r0,
                                           int& n, int& bank) {
  r0 = group_offsets[g];
  n = group_offsets[g + 1] - r0;
  if (n <= 0) return false;
  bank = group_bank_row[g];
  if (bank < 0 || bank >= bank_rows) {
    if (threadIdx.x == 0) record_error(err_word, LM_DEVERR_BAD_GROUP);
    return false;
  }
  return true;
}

// Offload variant: per group, the weight source from lm_slot_plan's table (slot, host store
// row written through into a slot, or host store row only).
struct OffloadSrc {
  const int32_t* group_src;     // per group: slot | LM_SRC_MISS flag, or LM_SRC_HOST
  const int32_t* group_expert;  // per group: expert id (host store row)
  const uint16_t* host;         // host store (device-visible pinned memory), expert-major
  uint16_t* slots;              // slot bank, slot-major
  int32_t num_slots;
  int32_t num_experts;
};

// Resolves group g's weight base for the offload variant; false (and an error word) on a
// malformed entry.
__device__ __forceinline__ bool offload_base(const OffloadSrc& off, int g, int64_t mat_elems,
                                             int32_t* err_word, const uint16_t*& wbase,
                                             uint16_t*& cbase, bool& sys) {
  const int code = off.group_src[g];
  const int e = off.group_expert[g];
  cbase = nullptr;
  if (code == LM_SRC_HOST || (code >= 0 && (code & LM_SRC_MISS))) {
    const int s = code == LM_SRC_HOST ? -1 : (code & ~LM_SRC_MISS);
    if (e < 0 || e >= off.num_experts || s >= off.num_slots) {
      if (threadIdx.x == 0) record_error(err_word, LM_DEVERR_BAD_GROUP);
      return false;
    }
    wbase = off.host + static_cast<int64_t>(e) * mat_elems;
    if (s >= 0) cbase = off.slots + static_cast<int64_t>(s) * mat_elems;
    sys = true;
    return true;
  }
  if (code < 0 || code >= off.num_slots) {
    if (threadIdx.x == 0) record_error(err_word, LM_DEVERR_UNMAPPED_EXPERT);
    return false;
  }
  wbase = off.slots + static_cast<int64_t>(code) * mat_elems;
  sys = false;
  return true;
}

template <int NC, bool OFFLOAD = false>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_gate_up_kernel(const uint16_t* __restrict__ hidden, int top_k,
                        const int32_t* __restrict__ row_to_pair,
                        const int32_t* __restrict__ group_offsets,
                        const int32_t* __restrict__ group_bank_row, int group_begin,
                        const uint16_t* __restrict__ w13_bank, int64_t bank_rows, int H, int I,
                        uint16_t* __restrict__ act, int32_t* __restrict__ err_word,
                        const OffloadSrc off = {}) {
  const int g = group_begin + blockIdx.x;
  int r0, n, bank = 0;
  const uint16_t* wbase;
  WeightSrc src{false, nullptr, nullptr};
  uint16_t* cbase = nullptr;
  if constexpr (OFFLOAD) {
    r0 = group_offsets[g];
    n = group_offsets[g + 1] - r0;
    if (n <= 0 || !offload_base(off, g, static_cast<int64_t>(2) * I * H, err_word, wbase, cbase,
                                src.sys))
      return;
  } else {
    if (!load_group(group_offsets, group_bank_row, g, bank_rows, err_word, r0, n, bank)) return;
    wbase = w13_bank + static_cast<int64_t>(bank) * 2 * I * H;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
  const int j0 = (blockIdx.y * kGemvWarps + warp) * 8;
  if (j0 >= I) return;
  const uint16_t* w_lo = wbase + tiled_row_base(j0 + gq, H);      // gate row
  const uint16_t* w_hi = wbase + tiled_row_base(I + j0 + gq, H);  // up row
  if (cbase != nullptr) {
    src.c_lo = cbase + tiled_row_base(j0 + gq, H);
    src.c_hi = cbase + tiled_row_base(I + j0 + gq, H);
  }
  for (int t0 = 0; t0 < n; t0 += 8 * NC) {
    const uint16_t* xrow[NC];
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      const int tok = t0 + q * 8 + gq;
      xrow[q] = (tok < n)
                    ? hidden + static_cast<int64_t>(row_to_pair[r0 + tok] / top_k) * H
                    : nullptr;
    }
    float acc[NC][4];
#pragma unroll
    for (int q = 0; q < NC; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
    warp_tile<NC, OFFLOAD>(w_lo, w_hi, xrow, H, acc, src);
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      const int ta = t0 + q * 8 + 2 * c;
      if (ta < n)
        act[static_cast<int64_t>(r0 + ta) * I + j0 + gq] =
            f32_to_bf16_bits(silu_f32(acc[q][0]) * acc[q][2]);
      if (ta + 1 < n)
        act[static_cast<int64_t>(r0 + ta + 1) * I + j0 + gq] =
            f32_to_bf16_bits(silu_f32(acc[q][1]) * acc[q][3]);
    }
  }
}

template <int NC, bool OFFLOAD = false>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_down_kernel(const uint16_t* __restrict__ act, const int32_t* __restrict__ group_offsets,
                     const int32_t* __restrict__ group_bank_row, int group_begin,
                     const uint16_t* __restrict__ w2_bank, int64_t bank_rows, int H, int I,
                     uint16_t* __restrict__ y_perm, int32_t* __restrict__ err_word,
                     const OffloadSrc off = {}) {
  const int g = group_begin + blockIdx.x;
  int r0, n, bank = 0;
  const uint16_t* wbase;
  WeightSrc src{false, nullptr, nullptr};
  uint16_t* cbase = nullptr;
  if constexpr (OFFLOAD) {
    r0 = group_offsets[g];
    n = group_offsets[g + 1] - r0;
    if (n <= 0 || !offload_base(off, g, static_cast<int64_t>(H) * I, err_word, wbase, cbase,
                                src.sys))
      return;
  } else {
    if (!load_group(group_offsets, group_bank_row, g, bank_rows, err_word, r0, n, bank)) return;
    wbase = w2_bank + static_cast<int64_t>(bank) * H * I;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
  const int n0 = (blockIdx.y * kGemvWarps + warp) * 16;
  if (n0 >= H) return;
  const uint16_t* w_lo = wbase + tiled_row_base(n0 + gq, I);
  const uint16_t* w_hi = wbase + tiled_row_base(n0 + 8 + gq, I);
  if (cbase != nullptr) {
    src.c_lo = cbase + tiled_row_base(n0 + gq, I);
    src.c_hi = cbase + tiled_row_base(n0 + 8 + gq, I);
  }
  for (int t0 = 0; t0 < n; t0 += 8 * NC) {
    const uint16_t* xrow[NC];
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      const int tok = t0 + q * 8 + gq;
      xrow[q] = (tok < n) ? act + static_cast<int64_t>(r0 + tok) * I : nullptr;
    }
    float acc[NC][4];
#pragma unroll
    for (int q = 0; q < NC; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
    warp_tile<NC, OFFLOAD>(w_lo, w_hi, xrow, I, acc, src);
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      const int ta = t0 + q * 8 + 2 * c;
      if (ta < n) {
        uint16_t* yr = y_perm + static_cast<int64_t>(r0 + ta) * H;
        yr[n0 + gq] = f32_to_bf16_bits(acc[q][0]);
        yr[n0 + 8 + gq] = f32_to_bf16_bits(acc[q][2]);
      }
      if (ta + 1 < n) {
        uint16_t* yr = y_perm + static_cast<int64_t>(r0 + ta + 1) * H;
        yr[n0 + gq] = f32_to_bf16_bits(acc[q][1]);
        yr[n0 + 8 + gq] = f32_to_bf16_bits(acc[q][3]);
      }
    }
  }
}

// Register-streaming launch pair: the fallback for calls whose (group, pass) count or group
// count exceeds the persistent kernel's tables.
template <int NC>
int launch_decode(const uint16_t* hidden, int top_k, const int32_t* row_to_pair,
                  const int32_t* group_offsets, const int32_t* group_bank_row, int group_begin,
                  int num_groups, const uint16_t* w13_bank, const uint16_t* w2_bank,
                  int64_t bank_rows, int H, int I, uint16_t* act, uint16_t* y_perm,
                  int32_t* err_word, cudaStream_t s) {
  const dim3 block(kGemvWarps * 32);
  const dim3 grid1(num_groups, (I + kGemvWarps * 8 - 1) / (kGemvWarps * 8));
  gemv_gate_up_kernel<NC><<<grid1, block, 0, s>>>(hidden, top_k, row_to_pair, group_offsets,
                                                   group_bank_row, group_begin, w13_bank,
                                                   bank_rows, H, I, act, err_word);
  int rc = launch_status("lm_moe_mlp_decode: gate_up");
  if (rc) return rc;
  const dim3 grid2(num_groups, (H + kGemvWarps * 16 - 1) / (kGemvWarps * 16));
  gemv_down_kernel<NC><<<grid2, block, 0, s>>>(act, group_offsets, group_bank_row, group_begin,
                                                w2_bank, bank_rows, H, I, y_perm, err_word);
  return launch_status("lm_moe_mlp_decode: down");
}

// ------------------------------------------------------------ persistent decode MLP kernel
// Both GEMMs of the decode MLP in one persistent launch (three CTAs per SM: more CTAs with
// shallower rings stream faster than fewer with deeper ones, measured). The work is a queue
// of small items, claimed one at a time with an atomic counter:
//   gate_up item: 32 gate rows + the matching 32 up rows of one expert x one token pass
//                 (8 * NC tokens of the group), over all of K = H;
//   down item:    64 W2 rows of one expert x one token pass, over K = I.
// All gate_up items come first in the queue, so a CTA that runs out of work early takes the
// next item anywhere, and the tail of the launch is one small item, not a whole expert.
// A down item reads the activations its expert's gate_up items wrote: each finished
// gate_up warp adds one to the pass's counter (a release reduction) and the down
// item's producer waits, bounded, until the count is complete. Items are claimed in queue
// order and a CTA processes its items in claim order (it claims the next one only after
// its current item's wait), so every awaited gate_up item belongs to a running CTA that
// reaches it without waiting on anything later: the wait always ends.
//
// Per CTA: one producer warp and 4 consumer warps around a ring of stages. A stage covers
// two 64-wide K tiles: the weight boxes, loaded by TMA from the bank's 3D tile map with box
// depth two (gate_up: gate rows and, from a second lane, up rows, 8 KiB each; down: 16 KiB),
// 128-byte swizzled, plus the matching K slices of the pass's 8 * NC token rows, copied by
// all producer lanes with cp.async (zero-filled past the group's end or the last K tile) and
// swizzled the same way. The stage's full barrier completes when the TMA bytes have landed
// and all 32 lanes' copies have, so consumers read only shared memory. The producer also
// writes each stage's item description next to the ring, published by the same barrier.
//
// The queue counter, the per-pass counters and an exit count live in a static per-device
// pool of counter sets (one per stream, so launches on different streams never share
// one); the last CTA to finish resets its set, so every launch starts from zeros.
constexpr int kPdConsumers = 4;
constexpr int kPdThreads = (kPdConsumers + 1) * 32;
constexpr int kPdWeightBytes = 16384;  // per stage: 2 K tiles x 64 weight rows
constexpr int kPdMaxGroups = 2048;
constexpr int kPdMaxSlots = 2048;  // (group, pass) pairs per launch
constexpr int kPdCounterSets = 16;
constexpr int kPdSmallPairs = 16;  // at most this many pairs: the deep-ring configuration
constexpr int kPdFirst = 1, kPdLast = 2, kPdDown = 4, kPdExit = 8;

struct PdCounters {
  int32_t work;
  int32_t exited;
  int32_t done[kPdMaxSlots];
};

__device__ PdCounters g_pd_counters[kPdCounterSets];

struct PdMeta {
  int32_t r0;      // first row of the group
  int32_t n;       // rows of the group
  int32_t tok0;    // first row of the pass within the group
  int32_t row0;    // first weight row of the item (gate / W2 row index)
  int32_t kt;      // first K tile of the stage
  int32_t ktiles;  // K tiles of the item
  int32_t slot;    // (group, pass) index
  int32_t flags;
};

struct PdParams {
  CUtensorMap w13map;  // w13 bank tiles, box {64, 32, 2}
  CUtensorMap w2map;   // w2 bank tiles, box {64, 64, 2}
  const uint16_t* hidden;
  const int32_t* row_to_pair;
  const int32_t* group_offsets;
  const int32_t* group_bank_row;
  uint16_t* act;
  uint16_t* y_perm;
  int32_t* err_word;
  int64_t bank_rows;
  int32_t counter_set;
  int32_t group_begin;
  int32_t num_groups;
  int32_t top_k;
  int32_t H;
  int32_t I;
};

template <int NC>
__host__ __device__ constexpr int pd_stages() {
  return NC == 8 ? 2 : 3;  // three CTAs per SM (NC = 8: the x slices double the stage)
}

template <int NC>
__host__ __device__ constexpr int pd_stage_bytes() {
  return kPdWeightBytes + 2 * NC * 8 * 128;  // multiple of 1024: bases stay swizzle-aligned
}

template <int NC, int S>
constexpr int pd_smem_bytes(int num_groups) {
  return 1024 + S * pd_stage_bytes<NC>() + ((num_groups + 1) * 4 + 15) / 16 * 16;
}

__device__ __forceinline__ uint4 lds_swz(const uint8_t* box, int row, int chunk) {
  return *reinterpret_cast<const uint4*>(box + row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void red_release_add_gpu(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One queue item as the producer streams it. xrow[j]: the token row behind the lane's j-th
// copied row (gate_up: the pair index, divided by top_k at use; down: the act row), or -1.
template <int NC>
struct PdItem {
  int w;  // queue index; >= the item count: the queue is exhausted
  int slot, row0, r0, n, bank, tok0;
  bool down;
  int xrow[2 * NC];
};

// Resolves queue index w (all producer lanes; lane l fills the rows it copies).
template <int NC>
__device__ __forceinline__ void pd_resolve(const PdParams& p, const int32_t* slot_prefix, int G,
                                           int w, int items, int items_gu, int tiles_gu,
                                           int tiles_dn, int lane, PdItem<NC>& it) {
  it.w = w;
  if (w >= items) return;
  it.down = w >= items_gu;
  const int wi = it.down ? w - items_gu : w;
  const int tiles = it.down ? tiles_dn : tiles_gu;
  it.slot = wi / tiles;
  const int tile = wi - it.slot * tiles;
  // group of the slot: the last g with slot_prefix[g] <= slot
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (slot_prefix[mid] <= it.slot) lo = mid; else hi = mid - 1;
  }
  it.r0 = p.group_offsets[p.group_begin + lo];
  it.n = p.group_offsets[p.group_begin + lo + 1] - it.r0;
  it.bank = p.group_bank_row[p.group_begin + lo];
  it.tok0 = (it.slot - slot_prefix[lo]) * 8 * NC;
  it.row0 = tile * (it.down ? 64 : 32);
#pragma unroll
  for (int j = 0; j < 2 * NC; ++j) {
    const int tok = it.tok0 + j * 4 + (lane >> 3);
    it.xrow[j] = tok >= it.n ? -1 : (it.down ? it.r0 + tok : p.row_to_pair[it.r0 + tok]);
  }
}

template <int NC, int S>
__global__ void __launch_bounds__(kPdThreads)
    gemv_persistent_kernel(const __grid_constant__ PdParams p) {
  constexpr int kStage = pd_stage_bytes<NC>();
  constexpr int kXSlice = NC * 8 * 128;  // one K tile of the pass's token rows
  constexpr int kLaneRows = NC * 2;      // token rows one producer lane copies per K tile
  constexpr int kPassRows = 8 * NC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  int32_t* slot_prefix = reinterpret_cast<int32_t*>(ring + S * kStage);  // [num_groups + 1]
  __shared__ uint64_t full[S], empty[S];
  __shared__ PdMeta meta[S];
  __shared__ int abort_flag;
  PdCounters* ctr = &g_pd_counters[p.counter_set];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.num_groups;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + 32);  // lane 0's arrival + 32 lanes' copy arrivals
      mbar_init(&empty[s], kPdConsumers);
    }
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  volatile int* ab = &abort_flag;
  // launched while the grouping drains: the work queue, the tables, the tokens and the
  // outputs are all touched only after this
  pdl_wait();

  if (warp == kPdConsumers) {
    // ---------------------------------------------------------------- producer
    // first item claimed at once, its latency hidden behind the table loads
    int w_first = 0;
    if (lane == 0) w_first = atomicAdd(&ctr->work, 1);
    // (group, pass) slots: slot_prefix[g] = slots of the groups before g. Empty groups and
    // groups with an out-of-range bank row get none (the latter also set the error word).
    int run = 0;
    for (int base = 0; base < G; base += 128) {
      // lane l: groups base + 4 l .. base + 4 l + 3, all table loads issued before any use
      const int g0 = base + lane * 4;
      int o[5], bk[4];
#pragma unroll
      for (int u = 0; u < 5; ++u)
        o[u] = g0 + u <= G ? p.group_offsets[p.group_begin + g0 + u] : 0;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        bk[u] = g0 + u < G ? p.group_bank_row[p.group_begin + g0 + u] : 0;
      int ps[4], tot = 0;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int n = o[u + 1] - o[u];
        ps[u] = 0;
        if (g0 + u < G && n > 0) {
          if (bk[u] < 0 || bk[u] >= p.bank_rows)
            record_error(p.err_word, LM_DEVERR_BAD_GROUP);
          else
            ps[u] = (n + kPassRows - 1) / kPassRows;
        }
        tot += ps[u];
      }
      int incl = tot;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
      }
      int excl = run + incl - tot;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (g0 + u < G) slot_prefix[g0 + u] = excl;
        excl += ps[u];
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) slot_prefix[G] = run;
    __syncwarp();
    // more (group, pass) pairs than counters (max_rows_per_group understated the groups):
    // nothing is computed and the error word says so
    const bool fits = run <= kPdMaxSlots;
    if (!fits) record_error(p.err_word, LM_DEVERR_BAD_GROUP);
    const int slots = fits ? run : 0;
    const int tiles_gu = p.I / 32, tiles_dn = p.H / 64;
    const int items_gu = slots * tiles_gu;
    const int items = items_gu + slots * tiles_dn;
    const int kt_gu = p.H >> 6, kt_dn = p.I >> 6;
    const int xchunk = lane & 7;
    if (lane == 0) {
      tma_prefetch_desc(&p.w13map);
      tma_prefetch_desc(&p.w2map);
    }
    int i = 0;  // stages issued
    bool ok = true;
    // The next item is claimed halfway through the current one and resolved (group lookup,
    // token rows) at its last stage, so neither the queue atomic nor the table loads stall
    // the ring; a CTA holds at most one item beyond the one it streams.
    PdItem<NC> cur;
    pd_resolve<NC>(p, slot_prefix, G, __shfl_sync(0xffffffffu, w_first, 0), items, items_gu,
                   tiles_gu, tiles_dn, lane, cur);
    while (ok && cur.w < items) {
      const bool down = cur.down;
      const int K = down ? p.I : p.H;
      const int ktiles = down ? kt_dn : kt_gu;
      if (down) {
        // wait until the pass's gate_up items have all written their activations
        const int need = tiles_gu * kPdConsumers;
        bool ready = true;
        if (lane == 0) {
          const long long t0 = clock64();
          while (ld_acquire_gpu(&ctr->done[cur.slot]) < need) {
            if (*ab || clock64() - t0 > LM_SPIN_LIMIT_CYCLES) {
              record_error(p.err_word, LM_DEVERR_WAIT_TIMEOUT);
              *ab = 1;
              ready = false;
              break;
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, ready, 0)) break;
        (void)ld_acquire_gpu(&ctr->done[cur.slot]);  // every copying lane acquires
      }
      const uint16_t* xsrc[kLaneRows];
#pragma unroll
      for (int j = 0; j < kLaneRows; ++j) {
        const int src = cur.xrow[j];
        xsrc[j] = src < 0 ? nullptr
                          : (down ? p.act : p.hidden) +
                                static_cast<int64_t>(down ? src : src / p.top_k) * K;
      }
      const int64_t zbase = (static_cast<int64_t>(cur.bank) *
                                 (down ? (p.H >> 7) : (2 * p.I) >> 7) +
                             (cur.row0 >> 7)) * ktiles;
      const int64_t zup = (static_cast<int64_t>(cur.bank) * ((2 * p.I) >> 7) +
                           ((p.I + cur.row0) >> 7)) * ktiles;
      const int kpairs = (ktiles + 1) >> 1;
      int w_next = 0;
      PdItem<NC> nxt;
      for (int kp = 0; kp < kpairs; ++kp, ++i) {
        const int st = i % S;
        const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&empty[st], ph ^ 1u, p.err_word, ab))) {
          ok = false;
          break;
        }
        uint8_t* dst = ring + st * kStage;
        const int kt = 2 * kp;
        if (lane == 0) {
          PdMeta m;
          m.r0 = cur.r0;
          m.n = cur.n;
          m.tok0 = cur.tok0;
          m.row0 = cur.row0;
          m.kt = kt;
          m.ktiles = ktiles;
          m.slot = cur.slot;
          m.flags = (kp == 0 ? kPdFirst : 0) | (kp == kpairs - 1 ? kPdLast : 0) |
                    (down ? kPdDown : 0);
          meta[st] = m;
          mbar_arrive_expect_tx(&full[st], kPdWeightBytes);
        }
        __syncwarp();
        const int la = (2 * i) & 31;
        if (down) {
          if (lane == la)
            tma_load_3d(dst, &p.w2map, &full[st], 0, cur.row0 & 127,
                        static_cast<int>(zbase + kt));
        } else if (lane == la) {
          tma_load_3d(dst, &p.w13map, &full[st], 0, cur.row0 & 127,
                      static_cast<int>(zbase + kt));
        } else if (lane == la + 1) {
          tma_load_3d(dst + kPdWeightBytes / 2, &p.w13map, &full[st], 0,
                      (p.I + cur.row0) & 127, static_cast<int>(zup + kt));
        }
        uint8_t* xs = dst + kPdWeightBytes;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const bool kin = kt + kk < ktiles;
#pragma unroll
          for (int j = 0; j < kLaneRows; ++j) {
            const int row = j * 4 + (lane >> 3);
            const bool v = kin && xsrc[j] != nullptr;
            cp_async_16(xs + kk * kXSlice + row * 128 + ((xchunk ^ (row & 7)) << 4),
                        v ? xsrc[j] + (kt + kk) * 64 + xchunk * 8 : p.hidden, v ? 16u : 0u);
          }
        }
        cp_async_arrive_noinc(&full[st]);
        if (kp == kpairs / 2 && lane == 0) w_next = atomicAdd(&ctr->work, 1);
        if (kp == kpairs - 1)
          pd_resolve<NC>(p, slot_prefix, G, __shfl_sync(0xffffffffu, w_next, 0), items,
                         items_gu, tiles_gu, tiles_dn, lane, nxt);
      }
      if (!ok) break;
      cur = nxt;
    }
    // this CTA claims nothing more: the next kernel (the combine) may start launching once
    // every CTA is here
    pdl_trigger();
    if (ok && !*ab) {
      // exit stage: consumers stop when they reach it
      const int st = i % S;
      const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
      if (__all_sync(0xffffffffu, mbar_wait_bounded(&empty[st], ph ^ 1u, p.err_word, ab))) {
        if (lane == 0) {
          meta[st].flags = kPdExit;
          mbar_arrive(&full[st]);
        }
        cp_async_arrive_noinc(&full[st]);
      }
    } else if (lane == 0) {
      // gave up: let the loads already issued land before the CTA can exit
      for (int j = i - S > 0 ? i - S : 0; j < i; ++j) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&full[j % S], static_cast<uint32_t>(j / S) & 1u) &&
               clock64() - t0 < 2000000) {
        }
      }
    }
    cp_async_wait_all();
  } else {
    // ---------------------------------------------------------------- consumers
    const int gq = lane >> 2, c = lane & 3;
    // independent accumulator chains (one per K block while registers allow) so that the
    // MMAs of a stage do not wait on one another
    constexpr int CH = NC <= 2 ? 2 : 1;
    float acc[CH][NC][4];
    for (int i = 0;; ++i) {
      const int st = i % S;
      const uint32_t ph = static_cast<uint32_t>(i / S) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[st], ph, p.err_word, ab))) break;
      const PdMeta m = meta[st];
      if (m.flags & kPdExit) break;
      const bool down = (m.flags & kPdDown) != 0;
      if (m.flags & kPdFirst) {
#pragma unroll
        for (int h = 0; h < CH; ++h)
#pragma unroll
          for (int q = 0; q < NC; ++q) acc[h][q][0] = acc[h][q][1] = acc[h][q][2] = acc[h][q][3] = 0.f;
      }
      const uint8_t* stage = ring + st * kStage;
      // gate_up: lo = gate row 8 warp + gq of the gate box, hi = the same row of the up box;
      // down: lo / hi = rows 16 warp + gq and 16 warp + 8 + gq of the 64-row box.
      const int lo_row = down ? 16 * warp + gq : 8 * warp + gq;
      const int hi_row = down ? lo_row + 8 : lo_row;
      const int ksub = down ? 8192 : 4096;
      const int hi_off = down ? 0 : kPdWeightBytes / 2;
      const int nk = m.kt + 1 < m.ktiles ? 2 : 1;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        if (kk < nk) {
          const uint8_t* box = stage + kk * ksub;
          const uint8_t* xs = stage + kPdWeightBytes + kk * kXSlice;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            const int h = (kk * 2 + kb) % CH;
            const uint4 wl = lds_swz(box, lo_row, kb * 4 + c);
            const uint4 wh = lds_swz(box + hi_off, hi_row, kb * 4 + c);
#pragma unroll
            for (int q = 0; q < NC; ++q) {
              const uint4 xv = lds_swz(xs, q * 8 + gq, kb * 4 + c);
              mma_16816(acc[h][q], wl.x, wh.x, wl.y, wh.y, xv.x, xv.y);
              mma_16816(acc[h][q], wl.z, wh.z, wl.w, wh.w, xv.z, xv.w);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (!(m.flags & kPdLast)) continue;
#pragma unroll
      for (int h = 1; h < CH; ++h)
#pragma unroll
        for (int q = 0; q < NC; ++q)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[0][q][e] += acc[h][q][e];
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        const int ta = m.tok0 + q * 8 + 2 * c;
        if (!down) {
          const int j = m.row0 + 8 * warp + gq;
          if (ta < m.n)
            p.act[static_cast<int64_t>(m.r0 + ta) * p.I + j] =
                f32_to_bf16_bits(silu_f32(acc[0][q][0]) * acc[0][q][2]);
          if (ta + 1 < m.n)
            p.act[static_cast<int64_t>(m.r0 + ta + 1) * p.I + j] =
                f32_to_bf16_bits(silu_f32(acc[0][q][1]) * acc[0][q][3]);
        } else {
          const int n0 = m.row0 + 16 * warp;
          if (ta < m.n) {
            uint16_t* yr = p.y_perm + static_cast<int64_t>(m.r0 + ta) * p.H;
            yr[n0 + gq] = f32_to_bf16_bits(acc[0][q][0]);
            yr[n0 + 8 + gq] = f32_to_bf16_bits(acc[0][q][2]);
          }
          if (ta + 1 < m.n) {
            uint16_t* yr = p.y_perm + static_cast<int64_t>(m.r0 + ta + 1) * p.H;
            yr[n0 + gq] = f32_to_bf16_bits(acc[0][q][1]);
            yr[n0 + 8 + gq] = f32_to_bf16_bits(acc[0][q][3]);
          }
        }
      }
      if (!down) {
        // the warp's activation stores, then one release increment of the pass's counter
        __syncwarp();
        if (lane == 0) red_release_add_gpu(&ctr->done[m.slot], 1);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&ctr->exited, 1) == static_cast<int>(gridDim.x) - 1) {
      // last CTA: every other CTA has finished with the counters
      const int slots = min(slot_prefix[G], kPdMaxSlots);
      for (int s = 0; s < slots; ++s) atomicExch(&ctr->done[s], 0);
      atomicExch(&ctr->work, 0);
      __threadfence();
      atomicExch(&ctr->exited, 0);
    }
  }
}

// Counter-set registry, per device. A stream keeps its set while it launches the persistent
// kernel. When every set is taken, a set whose stream's last eager launch has completed (an
// event recorded after each launch) moves to the new stream; a set launched inside a stream
// capture stays with its stream for good, since the graph replays it later. Only when no set
// can be freed does a launch take the register-streaming pair, and that is counted
// (lm_decode_counter_sets) and reported once on stderr.
struct PdSetEntry {
  cudaStream_t stream = nullptr;
  cudaEvent_t last = nullptr;  // recorded after the stream's latest eager launch
  bool used = false;
  bool pinned = false;  // launched during capture: never moves
  bool launched = false;
};
std::mutex g_pd_mu;
PdSetEntry g_pd_sets[64][kPdCounterSets];
long long g_pd_recycled = 0;
long long g_pd_fallbacks = 0;

bool stream_capturing(cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) != cudaSuccess) return true;  // unknown: treat as captured
  return st != cudaStreamCaptureStatusNone;
}

// -1: no set (take the two-kernel path)
int pd_counter_set(cudaStream_t s, bool capturing) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  std::lock_guard<std::mutex> lk(g_pd_mu);
  PdSetEntry* sets = g_pd_sets[dev];
  int free_set = -1;
  for (int i = 0; i < kPdCounterSets; ++i) {
    if (sets[i].used && sets[i].stream == s) return i;
    if (!sets[i].used && free_set < 0) free_set = i;
  }
  if (free_set < 0 && !capturing) {
    // a set whose owner's last eager launch has finished can move (no event query while
    // this stream captures: the query is not allowed there)
    for (int i = 0; i < kPdCounterSets && free_set < 0; ++i) {
      if (sets[i].pinned || sets[i].last == nullptr) continue;
      const cudaError_t q = sets[i].launched ? cudaEventQuery(sets[i].last) : cudaSuccess;
      if (q == cudaSuccess) {
        free_set = i;
        ++g_pd_recycled;
      } else if (cudaPeekAtLastError() == q) {
        (void)cudaGetLastError();  // not-ready is a status, not this launch's error
      }
    }
  }
  if (free_set < 0) {
    if (g_pd_fallbacks++ == 0)
      fprintf(stderr,
              "latchmoe_b200: lm_moe_mlp_decode: all %d counter sets of device %d are held by "
              "other streams (captured graphs or launches in flight); this and later such "
              "launches take the two-kernel decode path\n",
              kPdCounterSets, dev);
    return -1;
  }
  PdSetEntry& e = sets[free_set];
  if (e.last == nullptr &&
      cudaEventCreateWithFlags(&e.last, cudaEventDisableTiming) != cudaSuccess) {
    (void)cudaGetLastError();
    e.last = nullptr;
  }
  e.stream = s;
  e.used = true;
  e.pinned = false;
  e.launched = false;
  return free_set;
}

// After a launch with counter set `set` on stream s: pin it (capture) or record its event.
void pd_counter_set_launched(int set, cudaStream_t s, bool capturing) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lk(g_pd_mu);
  PdSetEntry& e = g_pd_sets[dev][set];
  if (capturing || e.last == nullptr) {
    e.pinned = true;  // no event to tell when it is free: keep it
    return;
  }
  if (cudaEventRecord(e.last, s) == cudaSuccess) {
    e.launched = true;
  } else {
    (void)cudaGetLastError();
    e.pinned = true;
  }
}

template <int NC, int S>
int launch_persistent(const uint16_t* hidden, int top_k, const int32_t* row_to_pair,
                             const int32_t* group_offsets, const int32_t* group_bank_row,
                             int group_begin, int num_groups, int max_rows,
                             const uint16_t* w13_bank, const uint16_t* w2_bank,
                             int64_t bank_rows, int H, int I, uint16_t* act, uint16_t* y_perm,
                             int32_t* err_word, int per_sm_cap, cudaStream_t s) {
  const int max_passes = (max_rows + 8 * NC - 1) / (8 * NC);
  const bool capturing = stream_capturing(s);
  const int set = (num_groups > kPdMaxGroups ||
                   static_cast<int64_t>(num_groups) * max_passes > kPdMaxSlots)
                      ? -1
                      : pd_counter_set(s, capturing);
  if (num_groups > kPdMaxGroups || static_cast<int64_t>(num_groups) * max_passes > kPdMaxSlots ||
      set < 0)
    return launch_decode<NC>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                             group_begin, num_groups, w13_bank, w2_bank, bank_rows, H, I, act,
                             y_perm, err_word, s);
  struct DevInfo {
    bool attr = false;
    int grid = 0;
  };
  static DevInfo info[64];
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "lm_moe_mlp_decode: device");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(LM_ERR_CUDA, "lm_moe_mlp_decode: device index");
  if (!info[dev].attr) {
    rc = check_cuda(cudaFuncSetAttribute(gemv_persistent_kernel<NC, S>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pd_smem_bytes<NC, S>(kPdMaxGroups)),
                    "lm_moe_mlp_decode: smem attribute");
    if (rc) return rc;
    int sms = 0, per_sm = 0;
    rc = check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                    "lm_moe_mlp_decode: SM count");
    if (rc) return rc;
    rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                        &per_sm, gemv_persistent_kernel<NC, S>, kPdThreads,
                        pd_smem_bytes<NC, S>(kPdMaxGroups)),
                    "lm_moe_mlp_decode: occupancy");
    if (rc) return rc;
    info[dev].grid = sms * (per_sm < 1 ? 1 : (per_sm > per_sm_cap ? per_sm_cap : per_sm));
    info[dev].attr = true;
  }
  PdParams prm{};
  rc = make_map(&prm.w13map, w13_bank, 3,
                static_cast<uint64_t>(bank_rows) * (2 * I / 128) * (H / 64), 0, 32, 2);
  if (rc) return rc;
  rc = make_map(&prm.w2map, w2_bank, 3,
                static_cast<uint64_t>(bank_rows) * (H / 128) * (I / 64), 0, 64, 2);
  if (rc) return rc;
  prm.hidden = hidden;
  prm.row_to_pair = row_to_pair;
  prm.group_offsets = group_offsets;
  prm.group_bank_row = group_bank_row;
  prm.act = act;
  prm.y_perm = y_perm;
  prm.err_word = err_word;
  prm.bank_rows = bank_rows;
  prm.counter_set = set;
  prm.group_begin = group_begin;
  prm.num_groups = num_groups;
  prm.top_k = top_k;
  prm.H = H;
  prm.I = I;
  const cudaError_t e =
      launch_dependent(gemv_persistent_kernel<NC, S>, dim3(info[dev].grid), dim3(kPdThreads),
                       pd_smem_bytes<NC, S>(num_groups), s, prm);
  if (e != cudaSuccess) return check_cuda(e, "lm_moe_mlp_decode: persistent");
  rc = launch_status("lm_moe_mlp_decode: persistent");
  if (rc == LM_OK) pd_counter_set_launched(set, s, capturing);
  return rc;
}

// Few pairs (batch 1 or 2): few items, each CTA streaming a long run, so deeper rings (5
// stages, two CTAs per SM) instead of three CTAs with three stages (measured at one token:
// 25 us vs 29.5 us for the 75 MB of its 8 experts).
template <int NC>
int launch_decode_persistent(const uint16_t* hidden, int top_k, const int32_t* row_to_pair,
                             const int32_t* group_offsets, const int32_t* group_bank_row,
                             int group_begin, int num_groups, int max_rows,
                             const uint16_t* w13_bank, const uint16_t* w2_bank,
                             int64_t bank_rows, int H, int I, uint16_t* act, uint16_t* y_perm,
                             int32_t* err_word, cudaStream_t s) {
  if (static_cast<int64_t>(max_rows) * top_k <= kPdSmallPairs)
    return launch_persistent<NC, 5>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                                    group_begin, num_groups, max_rows, w13_bank, w2_bank,
                                    bank_rows, H, I, act, y_perm, err_word, 2, s);
  return launch_persistent<NC, pd_stages<NC>()>(hidden, top_k, row_to_pair, group_offsets,
                                                group_bank_row, group_begin, num_groups,
                                                max_rows, w13_bank, w2_bank, bank_rows, H, I,
                                                act, y_perm, err_word, 3, s);
}

template <int NC>
int launch_decode_offload(const uint16_t* hidden, int top_k, const int32_t* row_to_pair,
                          const int32_t* group_offsets, int group_begin, int num_groups,
                          OffloadSrc o13, OffloadSrc o2, int H, int I, uint16_t* act,
                          uint16_t* y_perm, int32_t* err_word, cudaStream_t s) {
  const dim3 block(kGemvWarps * 32);
  const dim3 grid1(num_groups, (I + kGemvWarps * 8 - 1) / (kGemvWarps * 8));
  gemv_gate_up_kernel<NC, true><<<grid1, block, 0, s>>>(hidden, top_k, row_to_pair,
                                                         group_offsets, nullptr, group_begin,
                                                         nullptr, 0, H, I, act, err_word, o13);
  int rc = launch_status("lm_moe_mlp_decode_offload: gate_up");
  if (rc) return rc;
  const dim3 grid2(num_groups, (H + kGemvWarps * 16 - 1) / (kGemvWarps * 16));
  gemv_down_kernel<NC, true><<<grid2, block, 0, s>>>(act, group_offsets, nullptr, group_begin,
                                                      nullptr, 0, H, I, y_perm, err_word, o2);
  return launch_status("lm_moe_mlp_decode_offload: down");
}

// Device-visible address of pinned host memory (the same pointer on UVA systems), looked up
// once per (device, host pointer): later calls, including calls during stream capture, make
// no CUDA API call for it.
int device_alias(const void* host, const void** out, const char* what) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, const void*>, const void*>> cache;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), what);
  if (rc) return rc;
  {
    std::lock_guard<std::mutex> lk(mu);
    for (const auto& e : cache)
      if (e.first.first == dev && e.first.second == host) {
        *out = e.second;
        return LM_OK;
      }
  }
  void* d = nullptr;
  rc = check_cuda(cudaHostGetDevicePointer(&d, const_cast<void*>(host), 0), what);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() >= 1024) cache.erase(cache.begin());
  cache.push_back({{dev, host}, d});
  *out = d;
  return LM_OK;
}

}  // namespace
}  // namespace lm

using namespace lm;

extern "C" int lm_moe_mlp_decode_offload(
    const uint16_t* hidden, int32_t top_k, const int32_t* row_to_pair,
    const int32_t* group_offsets, const int32_t* group_src, const int32_t* group_expert,
    int32_t group_begin, int32_t group_end, int32_t max_rows_per_group,
    uint16_t* w13_slots, uint16_t* w2_slots, int32_t num_slots, const uint16_t* w13_host,
    const uint16_t* w2_host, int32_t num_experts, int32_t hidden_size, int32_t intermediate_size,
    uint16_t* act, uint16_t* y_perm, int32_t* err_word, void* stream) {
  const int H = hidden_size, I = intermediate_size;
  if (H <= 0 || I <= 0 || H % 128 != 0 || I % 64 != 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_mlp_decode_offload: need hidden_size % 128 == 0 and "
                "intermediate_size % 64 == 0 (tile-contiguous weight layout)");
  if (top_k <= 0 || group_begin < 0 || group_end < group_begin || num_slots <= 0 ||
      num_experts <= 0 || max_rows_per_group > 64)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_mlp_decode_offload: bad group range, sizes or more than 64 rows per group");
  if (group_end == group_begin) return LM_OK;
  if (hidden == nullptr || row_to_pair == nullptr || group_offsets == nullptr ||
      group_src == nullptr || group_expert == nullptr || w13_slots == nullptr ||
      w2_slots == nullptr || w13_host == nullptr || w2_host == nullptr || act == nullptr ||
      y_perm == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_decode_offload: null pointer");
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(w13_slots) |
       reinterpret_cast<uintptr_t>(w2_slots) | reinterpret_cast<uintptr_t>(w13_host) |
       reinterpret_cast<uintptr_t>(w2_host) | reinterpret_cast<uintptr_t>(act)) & 15)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_mlp_decode_offload: bases must be 16-byte aligned");
  const void* h13 = nullptr;
  const void* h2 = nullptr;
  int rc = device_alias(w13_host, &h13, "lm_moe_mlp_decode_offload: host w13 is not pinned");
  if (!rc) rc = device_alias(w2_host, &h2, "lm_moe_mlp_decode_offload: host w2 is not pinned");
  if (rc) return rc;
  const OffloadSrc o13{group_src, group_expert, static_cast<const uint16_t*>(h13), w13_slots,
                       num_slots, num_experts};
  const OffloadSrc o2{group_src, group_expert, static_cast<const uint16_t*>(h2), w2_slots,
                      num_slots, num_experts};
  const int ng = group_end - group_begin;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // One weight pass per group (<= 64 rows), so a missed expert crosses PCIe once.
  if (max_rows_per_group <= 8)
    return launch_decode_offload<1>(hidden, top_k, row_to_pair, group_offsets, group_begin, ng,
                                    o13, o2, H, I, act, y_perm, err_word, s);
  if (max_rows_per_group <= 16)
    return launch_decode_offload<2>(hidden, top_k, row_to_pair, group_offsets, group_begin, ng,
                                    o13, o2, H, I, act, y_perm, err_word, s);
  if (max_rows_per_group <= 32)
    return launch_decode_offload<4>(hidden, top_k, row_to_pair, group_offsets, group_begin, ng,
                                    o13, o2, H, I, act, y_perm, err_word, s);
  return launch_decode_offload<8>(hidden, top_k, row_to_pair, group_offsets, group_begin, ng,
                                  o13, o2, H, I, act, y_perm, err_word, s);
}

extern "C" int lm_decode_counter_sets(int32_t* in_use, int32_t* pinned, int64_t* recycled,
                                      int64_t* fallbacks) {
  int dev = 0;
  int rc = lm::check_cuda(cudaGetDevice(&dev), "lm_decode_counter_sets");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return lm::fail(LM_ERR_CUDA, "lm_decode_counter_sets: device");
  std::lock_guard<std::mutex> lk(lm::g_pd_mu);
  int u = 0, p = 0;
  for (const auto& e : lm::g_pd_sets[dev]) {
    u += e.used;
    p += e.used && e.pinned;
  }
  if (in_use) *in_use = u;
  if (pinned) *pinned = p;
  if (recycled) *recycled = lm::g_pd_recycled;
  if (fallbacks) *fallbacks = lm::g_pd_fallbacks;
  return LM_OK;
}

extern "C" int lm_moe_mlp_decode(const uint16_t* hidden, int32_t top_k,
                                 const int32_t* row_to_pair, const int32_t* group_offsets,
                                 const int32_t* group_bank_row, int32_t group_begin,
                                 int32_t group_end, int32_t max_rows_per_group,
                                 const uint16_t* w13_bank, const uint16_t* w2_bank,
                                 int64_t bank_rows, int32_t hidden_size,
                                 int32_t intermediate_size, uint16_t* act, uint16_t* y_perm,
                                 int32_t* err_word, void* stream) {
  const int H = hidden_size, I = intermediate_size;
  if (H <= 0 || I <= 0 || H % 128 != 0 || I % 64 != 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_mlp_decode: need hidden_size % 128 == 0 and intermediate_size % 64 == 0 "
                "(tile-contiguous weight layout)");
  if (top_k <= 0 || group_begin < 0 || group_end < group_begin || bank_rows <= 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_decode: bad group range or top_k");
  if (group_end == group_begin) return LM_OK;
  if (hidden == nullptr || row_to_pair == nullptr || group_offsets == nullptr ||
      group_bank_row == nullptr || w13_bank == nullptr || w2_bank == nullptr ||
      act == nullptr || y_perm == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_decode: null pointer");
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(w13_bank) |
       reinterpret_cast<uintptr_t>(w2_bank) | reinterpret_cast<uintptr_t>(act)) & 15)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_decode: bases must be 16-byte aligned");
  const int ng = group_end - group_begin;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Token chunks per weight pass: a group with more rows takes several passes (adjacent in the
  // work queue, so the repeated weight tiles come from L2). Narrow passes measured fastest up
  // to 64 rows per group (64-token decode layer: 142 us at NC = 2 vs 272 us at NC = 8).
  if (max_rows_per_group <= 8)
    return launch_decode_persistent<1>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                                       group_begin, ng, max_rows_per_group, w13_bank, w2_bank,
                                       bank_rows, H, I, act, y_perm, err_word, s);
  if (max_rows_per_group <= 64)
    return launch_decode_persistent<2>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                                       group_begin, ng, max_rows_per_group, w13_bank, w2_bank,
                                       bank_rows, H, I, act, y_perm, err_word, s);
  return launch_decode_persistent<8>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                                     group_begin, ng, max_rows_per_group, w13_bank, w2_bank,
                                     bank_rows, H, I, act, y_perm, err_word, s);
}
