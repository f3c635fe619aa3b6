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
#include <mutex>
#include <utility>
#include <vector>

#include "lm_common.cuh"

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
  if (max_rows_per_group <= 8)
    return launch_decode<1>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                            group_begin, ng, w13_bank, w2_bank, bank_rows, H, I, act, y_perm,
                            err_word, s);
  if (max_rows_per_group <= 16)
    return launch_decode<2>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                            group_begin, ng, w13_bank, w2_bank, bank_rows, H, I, act, y_perm,
                            err_word, s);
  if (max_rows_per_group <= 32)
    return launch_decode<4>(hidden, top_k, row_to_pair, group_offsets, group_bank_row,
                            group_begin, ng, w13_bank, w2_bank, bank_rows, H, I, act, y_perm,
                            err_word, s);
  return launch_decode<8>(hidden, top_k, row_to_pair, group_offsets, group_bank_row, group_begin,
                          ng, w13_bank, w2_bank, bank_rows, H, I, act, y_perm, err_word, s);
}
