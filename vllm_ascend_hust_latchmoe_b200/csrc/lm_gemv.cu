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
template <int NC>
__device__ __forceinline__ void warp_tile(const uint16_t* __restrict__ w_lo,
                                          const uint16_t* __restrict__ w_hi,
                                          const uint16_t* const (&xrow)[NC], int klen,
                                          float (&acc)[NC][4]) {
  const int c8 = (threadIdx.x & 3) * 8;
  const int nblk = klen / 32;
  constexpr int U = 4;
  int kb = 0;
  for (; kb + U <= nblk; kb += U) {
    uint4 wl[U], wh[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      wl[u] = ld_stream_16(w_lo + tiled_kblock(kb + u) + c8);
      wh[u] = ld_stream_16(w_hi + tiled_kblock(kb + u) + c8);
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
    const uint4 wl = ld_stream_16(w_lo + tiled_kblock(kb) + c8);
    const uint4 wh = ld_stream_16(w_hi + tiled_kblock(kb) + c8);
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

template <int NC>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_gate_up_kernel(const uint16_t* __restrict__ hidden, int top_k,
                        const int32_t* __restrict__ row_to_pair,
                        const int32_t* __restrict__ group_offsets,
                        const int32_t* __restrict__ group_bank_row, int group_begin,
                        const uint16_t* __restrict__ w13_bank, int64_t bank_rows, int H, int I,
                        uint16_t* __restrict__ act, int32_t* __restrict__ err_word) {
  int r0, n, bank;
  if (!load_group(group_offsets, group_bank_row, group_begin + blockIdx.x, bank_rows, err_word,
                  r0, n, bank))
    return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
  const int j0 = (blockIdx.y * kGemvWarps + warp) * 8;
  if (j0 >= I) return;
  const uint16_t* wbase = w13_bank + static_cast<int64_t>(bank) * 2 * I * H;
  const uint16_t* w_lo = wbase + tiled_row_base(j0 + gq, H);      // gate row
  const uint16_t* w_hi = wbase + tiled_row_base(I + j0 + gq, H);  // up row
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
    warp_tile<NC>(w_lo, w_hi, xrow, H, acc);
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

template <int NC>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_down_kernel(const uint16_t* __restrict__ act, const int32_t* __restrict__ group_offsets,
                     const int32_t* __restrict__ group_bank_row, int group_begin,
                     const uint16_t* __restrict__ w2_bank, int64_t bank_rows, int H, int I,
                     uint16_t* __restrict__ y_perm, int32_t* __restrict__ err_word) {
  int r0, n, bank;
  if (!load_group(group_offsets, group_bank_row, group_begin + blockIdx.x, bank_rows, err_word,
                  r0, n, bank))
    return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
  const int n0 = (blockIdx.y * kGemvWarps + warp) * 16;
  if (n0 >= H) return;
  const uint16_t* wbase = w2_bank + static_cast<int64_t>(bank) * H * I;
  const uint16_t* w_lo = wbase + tiled_row_base(n0 + gq, I);
  const uint16_t* w_hi = wbase + tiled_row_base(n0 + 8 + gq, I);
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
    warp_tile<NC>(w_lo, w_hi, xrow, I, acc);
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

}  // namespace
}  // namespace lm

using namespace lm;

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
