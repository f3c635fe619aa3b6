// Prefill path of the grouped expert MLP on the 5th-generation tensor cores (tcgen05).
//
// One persistent kernel runs both GEMMs of the expert MLP (selected by `mode`):
//   mode 0 (gate_up): act[r, n0:n0+128] = silu(X_r . W13[n0:n0+128]) * (X_r . W13[I+n0:...])
//                     MMA N = 256 = 128 gate rows + the 128 matching up rows, so the fused
//                     SiLU*mul epilogue has both halves of every output column in TMEM.
//   mode 1 (down):    y[r, n0:n0+256] = act_r . W2[n0:n0+256]
// Tiles: 128 rows x 256 MMA columns x 64-wide K steps (one 128-byte swizzle row of bf16).
// Warp roles (192 threads): warp 0 issues TMA loads into a 4-stage smem ring, warp 1 issues
// tcgen05.mma into one of two TMEM accumulators (2 x 256 fp32 columns = all 512 columns),
// warps 2-5 drain the other accumulator (tcgen05.ld -> epilogue -> global stores), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
// Tiles are enumerated (group, m-tile, n-tile) with n fastest, so CTAs running at the same
// time share the A rows and the expert's weight tiles in L2. The tile list is derived on
// the device from group_offsets, so the launch itself is independent of the routing.
// No TMA load uses cluster multicast; every operand is this GPU's own memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

#include "lm_common.cuh"

namespace lm {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int MAX_G = 256;
constexpr int NUM_THREADS = 192;

struct SmemCtl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int mprefix[MAX_G + 1];
  int row0[MAX_G];
  int nrows[MAX_G];
  int bank[MAX_G];
};

constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + static_cast<int>(sizeof(SmemCtl));

struct UmmaParams {
  CUtensorMap tmap_a;  // A rows [R, K] bf16, box {64, 128}
  CUtensorMap tmap_b;  // weight bank [bank_rows, N_total, K], box {64, 128|256, 1}
  const int32_t* group_offsets;
  const int32_t* group_bank_row;
  uint16_t* out;
  int32_t* err_word;
  int32_t group_begin;
  int32_t num_groups;
  int32_t k_blocks;
  int32_t n_tiles;
  int32_t mode;
  int32_t inter;   // I: row offset of the up half inside W13 (mode 0)
  int32_t out_ld;  // output row stride (elements)
  int32_t bank_rows;
};

struct TileCoord {
  int g;      // local group index
  int row0;   // first A row of the tile
  int valid;  // rows of the tile that belong to the group
  int nt;     // n-tile index
};

__device__ __forceinline__ TileCoord decode_tile(const SmemCtl& c, int t, int n_tiles, int G) {
  const int mg = t / n_tiles;
  TileCoord tc;
  tc.nt = t - mg * n_tiles;
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (c.mprefix[mid] <= mg)
      lo = mid;
    else
      hi = mid - 1;
  }
  tc.g = lo;
  const int ml = mg - c.mprefix[lo];
  tc.row0 = c.row0[lo] + ml * BM;
  const int rem = c.nrows[lo] - ml * BM;
  tc.valid = rem < BM ? rem : BM;
  return tc;
}

__device__ __forceinline__ void store_row_chunk(uint16_t* dst, const uint32_t (&packed)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  d[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  d[2] = make_uint4(packed[8], packed[9], packed[10], packed[11]);
  d[3] = make_uint4(packed[12], packed[13], packed[14], packed[15]);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    umma_grouped_kernel(const __grid_constant__ UmmaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SmemCtl& c = *reinterpret_cast<SmemCtl*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.num_groups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&c.full[s], 1);
      mbar_init(&c.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&c.tfull[a], 1);
      mbar_init(&c.tempty[a], 4);
    }
    c.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&c.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = threadIdx.x; i < G; i += NUM_THREADS) {
    const int g = p.group_begin + i;
    const int r0 = p.group_offsets[g];
    int n = p.group_offsets[g + 1] - r0;
    int bank = p.group_bank_row[g];
    if (n > 0 && (bank < 0 || bank >= p.bank_rows)) {
      record_error(p.err_word, LM_DEVERR_BAD_GROUP);
      n = 0;
      bank = 0;
    }
    c.row0[i] = r0;
    c.nrows[i] = n > 0 ? n : 0;
    c.bank[i] = bank;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < G; base += 32) {
      const int i = base + lane;
      int v = (i < G) ? (c.nrows[i] + BM - 1) / BM : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (i < G) c.mprefix[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) c.mprefix[0] = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = c.tmem_base;
  const int total_tiles = c.mprefix[G] * p.n_tiles;
  volatile int* abort_flag = &c.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued_parity[STAGES];
      for (int s = 0; s < STAGES; ++s) issued_parity[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(c, t, p.n_tiles, G);
        const int bank = c.bank[tc.g];
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&c.empty[stage], phase ^ 1u, p.err_word, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&c.full[stage], STAGE_BYTES);
          tma_load_2d(sa, &p.tmap_a, &c.full[stage], kb * BK, tc.row0);
          if (p.mode == 0) {
            tma_load_3d(sb, &p.tmap_b, &c.full[stage], kb * BK, tc.nt * 128, bank);
            tma_load_3d(sb + B_BYTES / 2, &p.tmap_b, &c.full[stage], kb * BK,
                        p.inter + tc.nt * 128, bank);
          } else {
            tma_load_3d(sb, &p.tmap_b, &c.full[stage], kb * BK, tc.nt * BN, bank);
          }
          issued_parity[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s) {
          if (issued_parity[s] < 0) continue;
          const long long t0 = clock64();
          while (!mbar_try_wait(&c.full[s], static_cast<uint32_t>(issued_parity[s])) &&
                 clock64() - t0 < LM_SPIN_LIMIT_CYCLES) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        if (!mbar_wait_bounded(&c.tempty[acc], acc_phase ^ 1u, p.err_word, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&c.full[stage], phase, p.err_word, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            umma_bf16(d_tmem, sdesc_k_sw128(a_addr + kk * 32), sdesc_k_sw128(b_addr + kk * 32),
                      idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&c.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&c.tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue warps 2..5
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32) are visible to this warp
    const int r = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileCoord tc = decode_tile(c, t, p.n_tiles, G);
      if (!mbar_wait_bounded(&c.tfull[acc], acc_phase, p.err_word, abort_flag)) break;
      tc_fence_after();
      const bool valid = r < tc.valid;
      uint16_t* out_row = p.out + static_cast<int64_t>(tc.row0 + r) * p.out_ld;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (p.mode == 0) {
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t gv[32], uv[32];
          tmem_ld_32x32b_x32(tbase + ch * 32, gv);
          tmem_ld_32x32b_x32(tbase + 128 + ch * 32, uv);
          tmem_ld_wait();
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = silu_f32(__uint_as_float(gv[2 * i])) * __uint_as_float(uv[2 * i]);
            const float a1 =
                silu_f32(__uint_as_float(gv[2 * i + 1])) * __uint_as_float(uv[2 * i + 1]);
            packed[i] = pack_bf16x2(a0, a1);
          }
          if (valid) store_row_chunk(out_row + tc.nt * 128 + ch * 32, packed);
        }
      } else {
#pragma unroll 1
        for (int ch = 0; ch < 8; ++ch) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tbase + ch * 32, v);
          tmem_ld_wait();
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            packed[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          if (valid) store_row_chunk(out_row + tc.nt * BN + ch * 32, packed);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  uint64_t d[3];
  uint32_t box1;
  int rank;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && d[0] == o.d[0] && d[1] == o.d[1] && d[2] == o.d[2] &&
           box1 == o.box1 && rank == o.rank;
  }
};

struct MapCache {
  std::mutex mu;
  std::vector<std::pair<MapKey, CUtensorMap>> entries;
};

MapCache& map_cache() {
  static MapCache c;
  return c;
}

// rank 2: dims {K, rows}; rank 3: dims {K, N, bank_rows}. Box {64, box1(, 1)}, 128B swizzle.
int make_map(CUtensorMap* out, const void* ptr, int rank, uint64_t d0, uint64_t d1, uint64_t d2,
             uint32_t box1) {
  const MapKey key{ptr, {d0, d1, d2}, box1, rank};
  MapCache& cache = map_cache();
  {
    std::lock_guard<std::mutex> lk(cache.mu);
    for (auto& e : cache.entries)
      if (e.first == key) {
        *out = e.second;
        return LM_OK;
      }
  }
  auto fn = encode_fn();
  if (fn == nullptr) return fail(LM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(BK), box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap m;
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                        const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LM_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  {
    std::lock_guard<std::mutex> lk(cache.mu);
    if (cache.entries.size() >= 256) cache.entries.erase(cache.entries.begin());
    cache.entries.emplace_back(key, m);
  }
  *out = m;
  return LM_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

int ensure_smem_attr() {
  static int done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return LM_OK;
  int rc = check_cuda(cudaFuncSetAttribute(umma_grouped_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           SMEM_BYTES),
                      "lm_moe_mlp_prefill: smem attribute");
  if (rc == LM_OK && dev >= 0 && dev < 64) done[dev] = 1;
  return rc;
}

}  // namespace
}  // namespace lm

using namespace lm;

extern "C" int lm_moe_mlp_prefill(const uint16_t* x_perm, int64_t total_rows,
                                  const int32_t* group_offsets, const int32_t* group_bank_row,
                                  int32_t group_begin, int32_t group_end,
                                  const uint16_t* w13_bank, const uint16_t* w2_bank,
                                  int64_t bank_rows, int32_t hidden_size,
                                  int32_t intermediate_size, uint16_t* act, uint16_t* y_perm,
                                  int32_t* err_word, void* stream) {
  const int H = hidden_size, I = intermediate_size;
  if (H <= 0 || I <= 0 || H % BN != 0 || I % 128 != 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_mlp_prefill: need hidden_size % 256 == 0 and intermediate_size % 128 == 0");
  if (group_begin < 0 || group_end < group_begin || group_end - group_begin > MAX_G)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_moe_mlp_prefill: group range must hold at most 256 groups");
  if (bank_rows <= 0 || bank_rows > 0x7fffffff || total_rows < 0 || total_rows > 0x7fffffff)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_prefill: bad bank_rows or total_rows");
  if (group_end == group_begin || total_rows == 0) return LM_OK;
  if (x_perm == nullptr || group_offsets == nullptr || group_bank_row == nullptr ||
      w13_bank == nullptr || w2_bank == nullptr || act == nullptr || y_perm == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_prefill: null pointer");
  if ((reinterpret_cast<uintptr_t>(x_perm) | reinterpret_cast<uintptr_t>(w13_bank) |
       reinterpret_cast<uintptr_t>(w2_bank) | reinterpret_cast<uintptr_t>(act) |
       reinterpret_cast<uintptr_t>(y_perm)) & 15)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_prefill: bases must be 16-byte aligned");
  int rc = ensure_smem_attr();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = sm_count();

  UmmaParams p1{};
  rc = make_map(&p1.tmap_a, x_perm, 2, H, total_rows, 1, BM);
  if (rc) return rc;
  rc = make_map(&p1.tmap_b, w13_bank, 3, H, 2 * static_cast<uint64_t>(I), bank_rows, 128);
  if (rc) return rc;
  p1.group_offsets = group_offsets;
  p1.group_bank_row = group_bank_row;
  p1.out = act;
  p1.err_word = err_word;
  p1.group_begin = group_begin;
  p1.num_groups = group_end - group_begin;
  p1.k_blocks = H / BK;
  p1.n_tiles = I / 128;
  p1.mode = 0;
  p1.inter = I;
  p1.out_ld = I;
  p1.bank_rows = static_cast<int32_t>(bank_rows);
  umma_grouped_kernel<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(p1);
  rc = launch_status("lm_moe_mlp_prefill: gate_up");
  if (rc) return rc;

  UmmaParams p2 = p1;
  rc = make_map(&p2.tmap_a, act, 2, I, total_rows, 1, BM);
  if (rc) return rc;
  rc = make_map(&p2.tmap_b, w2_bank, 3, I, H, bank_rows, BN);
  if (rc) return rc;
  p2.out = y_perm;
  p2.k_blocks = I / BK;
  p2.n_tiles = H / BN;
  p2.mode = 1;
  p2.out_ld = H;
  umma_grouped_kernel<<<grid, NUM_THREADS, SMEM_BYTES, s>>>(p2);
  return launch_status("lm_moe_mlp_prefill: down");
}
