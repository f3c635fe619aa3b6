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
// Tile order: groups with several m-tiles ("heavy": their weight tiles are reused from L2,
// so their tiles are tensor-bound) and single-m-tile groups ("light": every weight tile is
// read from DRAM once, so their tiles are HBM-bound) form two lists, each enumerated
// (group, m-tile, n-tile) with n fastest, and the two lists are merged in proportion. CTAs
// running at the same time then mix both kinds, overlapping weight streaming with MMAs.
// The tile lists are derived on the device from group_offsets, so the launch itself is
// independent of the routing.
// No TMA load uses cluster multicast; every operand is this GPU's own memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "lm_common.cuh"

namespace lm {
namespace {

constexpr int BM = 128;   // rows per CTA (TMEM lanes)
constexpr int BN = 256;   // MMA N (mode 0: 128 gate + 128 up rows; mode 1: 256 outputs)
constexpr int BK = 64;    // one 128-byte swizzle row of bf16
constexpr int A_BYTES = BM * BK * 2;      // 16 KiB
constexpr int B_TILE_BYTES = 128 * BK * 2;  // one 128-row weight tile, 16 KiB
constexpr int TMEM_COLS = 512;
constexpr int MAX_G = 256;
constexpr int NUM_THREADS = 192;

// PAIR = 1: one CTA owns a 128-row tile and loads the whole 256-row B tile.
// PAIR = 2: a cluster of two CTAs owns a 256-row tile (M = 256, cta_group::2); each CTA
// loads its own 128 A rows and one 128-row half of B, the leader issues the MMAs.
template <int PAIR>
struct Cfg {
  static constexpr int STAGE_BYTES = A_BYTES + (PAIR == 1 ? 2 : 1) * B_TILE_BYTES;
  static constexpr int STAGES = PAIR == 1 ? 4 : 6;
  static constexpr int UNIT_ROWS = BM * PAIR;
};

struct SmemCtl {
  uint64_t full[6];
  uint64_t empty[6];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int hprefix[MAX_G + 1];  // unit-tiles of heavy groups before group i
  int lprefix[MAX_G + 1];  // light groups (exactly one unit-tile) before group i
  int row0[MAX_G];
  int nrows[MAX_G];
  int bank[MAX_G];
};

template <int PAIR>
constexpr int smem_bytes() {
  return 1024 + Cfg<PAIR>::STAGES * Cfg<PAIR>::STAGE_BYTES + static_cast<int>(sizeof(SmemCtl));
}

struct UmmaParams {
  CUtensorMap tmap_a;  // A rows [R, K] bf16, box {64, 128}
  CUtensorMap tmap_b;  // weight tiles [bank_rows * N/128 * K/64][128][64], box {64, 128, 1}
  const int32_t* group_offsets;
  const int32_t* group_bank_row;
  uint16_t* out;
  int32_t* err_word;
  int32_t group_begin;
  int32_t num_groups;
  int32_t k_blocks;
  int32_t n_tiles;
  int32_t mode;
  int32_t up_tile;   // mode 0: 128-row tile index of the first up row (I / 128)
  int32_t out_ld;    // output row stride (elements)
  int32_t bank_rows;
  int32_t w_ntiles;  // 128-row tiles per expert matrix (N / 128)
};

struct TileCoord {
  int g;      // local group index
  int row0;   // first A row of the unit tile
  int valid;  // rows of the unit tile that belong to the group
  int nt;     // n-tile index
};

// Largest i in [0, G) with prefix[i] <= v (prefix is non-decreasing, prefix[G] > v).
__device__ __forceinline__ int find_group(const int* prefix, int v, int G) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= v)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Position t of the merged order -> (group, unit-tile, n-tile). Heavy tiles before position
// t: floor(t * Th / T); t is heavy iff that count grows at t + 1.
__device__ __forceinline__ TileCoord decode_tile(const SmemCtl& c, int t, int n_tiles, int G,
                                                 int heavy_tiles, int total_tiles, int unit) {
  const long long th = heavy_tiles, tt = total_tiles;
  const int hb = static_cast<int>((static_cast<long long>(t) * th) / tt);
  const int hb1 = static_cast<int>((static_cast<long long>(t + 1) * th) / tt);
  TileCoord tc;
  int g, ml;
  if (hb1 > hb) {
    const int mg = hb / n_tiles;
    tc.nt = hb - mg * n_tiles;
    g = find_group(c.hprefix, mg, G);
    ml = mg - c.hprefix[g];
  } else {
    const int li = t - hb;
    const int mg = li / n_tiles;
    tc.nt = li - mg * n_tiles;
    g = find_group(c.lprefix, mg, G);
    ml = 0;
  }
  tc.g = g;
  tc.row0 = c.row0[g] + ml * unit;
  const int rem = c.nrows[g] - ml * unit;
  tc.valid = rem < unit ? rem : unit;
  return tc;
}

__device__ __forceinline__ void store_row_chunk(uint16_t* dst, const uint32_t (&packed)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  d[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  d[2] = make_uint4(packed[8], packed[9], packed[10], packed[11]);
  d[3] = make_uint4(packed[12], packed[13], packed[14], packed[15]);
}

template <int PAIR>
__device__ __forceinline__ void umma_grouped_body(const UmmaParams& p) {
  using C = Cfg<PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SmemCtl& c = *reinterpret_cast<SmemCtl*>(smem + C::STAGES * C::STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.num_groups;
  const uint32_t rank = PAIR == 2 ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x / PAIR;
  const int num_clusters = gridDim.x / PAIR;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&c.full[s], 1);
      mbar_init(&c.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&c.tfull[a], 1);
      mbar_init(&c.tempty[a], 4 * PAIR);
    }
    c.abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_b);
  }
  if (warp == 1) {
    if (PAIR == 2) {
      tmem_alloc_pair(&c.tmem_base, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&c.tmem_base, TMEM_COLS);
      tmem_relinquish();
    }
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
  if (warp < 2) {
    // warp 0: prefix of heavy unit-tiles; warp 1: prefix of light groups.
    int* prefix = warp == 0 ? c.hprefix : c.lprefix;
    int carry = 0;
    for (int base = 0; base < G; base += 32) {
      const int i = base + lane;
      const int mt = (i < G) ? (c.nrows[i] + C::UNIT_ROWS - 1) / C::UNIT_ROWS : 0;
      int v = warp == 0 ? (mt >= 2 ? mt : 0) : (mt == 1 ? 1 : 0);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (i < G) prefix[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) prefix[0] = 0;
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR == 2) cluster_sync_all();  // peer barriers initialised, both TMEM halves allocated
  tc_fence_after();

  const uint32_t tmem_base = c.tmem_base;
  const int heavy_tiles = c.hprefix[G] * p.n_tiles;
  const int total_tiles = heavy_tiles + c.lprefix[G] * p.n_tiles;
  volatile int* abort_flag = &c.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued_parity[6];
      for (int s = 0; s < 6; ++s) issued_parity[s] = -1;
      bool ok = true;
      for (int t = cluster_id; t < total_tiles && ok; t += num_clusters) {
        const TileCoord tc = decode_tile(c, t, p.n_tiles, G, heavy_tiles, total_tiles,
                                         C::UNIT_ROWS);
        // Tile index of (expert row, 128-row tile, k block) in the tile-contiguous bank.
        const int ebase = c.bank[tc.g] * p.w_ntiles;
        const int nt0 = p.mode == 0 ? tc.nt : 2 * tc.nt;
        const int nt1 = p.mode == 0 ? p.up_tile + tc.nt : 2 * tc.nt + 1;
        const int a_row = tc.row0 + static_cast<int>(rank) * BM;
        const int my_nt = rank == 0 ? nt0 : nt1;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&c.empty[stage], phase ^ 1u, p.err_word, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          if (PAIR == 1) {
            mbar_arrive_expect_tx(&c.full[stage], C::STAGE_BYTES);
            tma_load_2d(sa, &p.tmap_a, &c.full[stage], kb * BK, a_row);
            tma_load_3d(sb, &p.tmap_b, &c.full[stage], 0, 0, (ebase + nt0) * p.k_blocks + kb);
            tma_load_3d(sb + B_TILE_BYTES, &p.tmap_b, &c.full[stage], 0, 0,
                        (ebase + nt1) * p.k_blocks + kb);
          } else {
            // Both CTAs' bytes complete on the leader's barrier; only the leader arrives.
            const uint32_t full_leader = mapa_shared(smem_u32(&c.full[stage]), 0);
            if (leader) mbar_arrive_expect_tx(&c.full[stage], 2 * C::STAGE_BYTES);
            tma_load_2d_pair(sa, &p.tmap_a, full_leader, kb * BK, a_row);
            tma_load_3d_pair(sb, &p.tmap_b, full_leader, 0, 0, (ebase + my_nt) * p.k_blocks + kb);
          }
          issued_parity[stage] = static_cast<int>(phase);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Wait until the MMAs released every stage this CTA filled, so no TMA write or
      // commit arrival into this CTA's shared memory is still in flight at exit.
      for (int s = 0; s < C::STAGES; ++s) {
        if (issued_parity[s] < 0) continue;
        const long long t0 = clock64();
        while (!mbar_try_wait(&c.empty[s], static_cast<uint32_t>(issued_parity[s])) &&
               clock64() - t0 < LM_SPIN_LIMIT_CYCLES) {
          if (*abort_flag && clock64() - t0 > 200000) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(BM * PAIR, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster_id; t < total_tiles && ok; t += num_clusters) {
        if (!mbar_wait_bounded(&c.tempty[acc], acc_phase ^ 1u, p.err_word, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&c.full[stage], phase, p.err_word, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sdesc_k_sw128(a_addr + kk * 32);
            const uint64_t bd = sdesc_k_sw128(b_addr + kk * 32);
            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
            if (PAIR == 2)
              umma_bf16_pair(d_tmem, ad, bd, idesc, accum);
            else
              umma_bf16(d_tmem, ad, bd, idesc, accum);
          }
          if (PAIR == 2)
            umma_commit_pair(&c.empty[stage], 0x3);
          else
            umma_commit(&c.empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR == 2)
          umma_commit_pair(&c.tfull[acc], 0x3);
        else
          umma_commit(&c.tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue warps 2..5
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32) are visible to this warp
    const int r = quad * 32 + lane;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&c.tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&c.tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster_id; t < total_tiles; t += num_clusters) {
      const TileCoord tc = decode_tile(c, t, p.n_tiles, G, heavy_tiles, total_tiles,
                                       C::UNIT_ROWS);
      if (!mbar_wait_bounded(&c.tfull[acc], acc_phase, p.err_word, abort_flag)) break;
      tc_fence_after();
      const int my_valid = tc.valid - static_cast<int>(rank) * BM;
      const bool valid = r < my_valid;
      uint16_t* out_row =
          p.out + static_cast<int64_t>(tc.row0 + static_cast<int>(rank) * BM + r) * p.out_ld;
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
      if (lane == 0) {
        if (PAIR == 2)
          mbar_arrive_remote(acc == 0 ? tempty_leader0 : tempty_leader1);
        else
          mbar_arrive(&c.tempty[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR == 2) cluster_sync_all();  // both CTAs done with TMEM and with remote barriers
  if (warp == 1) {
    tc_fence_after();
    if (PAIR == 2)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    umma_grouped_kernel(const __grid_constant__ UmmaParams p) {
  umma_grouped_body<1>(p);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    umma_grouped_kernel_2sm(const __grid_constant__ UmmaParams p) {
  umma_grouped_body<2>(p);
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
  int rank;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && d[0] == o.d[0] && d[1] == o.d[1] && d[2] == o.d[2] && rank == o.rank;
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

// rank 2: activation rows, dims {K, rows}, box {64, 128}.
// rank 3: weight tiles, dims {64, 128, n_tiles} with strides {128 B, 16 KiB}, box {64, 128, 1}.
// Both with 128-byte swizzle (the K-major SW128 layout the UMMA descriptors expect).
int make_map(CUtensorMap* out, const void* ptr, int rank, uint64_t d0, uint64_t d1) {
  const MapKey key{ptr, {d0, d1, 0}, rank};
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
  cuuint64_t dims[3];
  cuuint64_t strides[2];
  if (rank == 2) {
    dims[0] = d0;
    dims[1] = d1;
    strides[0] = d0 * 2;
  } else {
    dims[0] = BK;
    dims[1] = 128;
    dims[2] = d0;  // number of 128 x 64 tiles
    strides[0] = BK * 2;
    strides[1] = BK * 128 * 2;
  }
  cuuint32_t box[3] = {static_cast<cuuint32_t>(BK), 128, 1};
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
                                           smem_bytes<1>()),
                      "lm_moe_mlp_prefill: smem attribute");
  if (rc) return rc;
  rc = check_cuda(cudaFuncSetAttribute(umma_grouped_kernel_2sm,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes<2>()),
                  "lm_moe_mlp_prefill: smem attribute (2-SM)");
  if (rc == LM_OK && dev >= 0 && dev < 64) done[dev] = 1;
  return rc;
}

// Single-CTA tiles by default: on Zipf-skewed expert loads most groups fit one 128-row
// tile, and a 256-row 2-SM tile would leave the second CTA's half empty for them (measured
// 409 us vs 453 us on the 4096-token Qwen3-30B-A3B layer). LM_UMMA_CTA_PAIR=2 selects the
// cta_group::2 tiles, which win on dense groups (1233 vs 1155 TFLOP/s on one 32768-row group).
int cta_pair() {
  static int v = [] {
    const char* e = getenv("LM_UMMA_CTA_PAIR");
    return (e != nullptr && e[0] == '2') ? 2 : 1;
  }();
  return v;
}

int launch_umma(const UmmaParams& p, int grid, cudaStream_t s, const char* what) {
  if (cta_pair() == 2) {
    umma_grouped_kernel_2sm<<<grid & ~1, NUM_THREADS, smem_bytes<2>(), s>>>(p);
  } else {
    umma_grouped_kernel<<<grid, NUM_THREADS, smem_bytes<1>(), s>>>(p);
  }
  return launch_status(what);
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
  rc = make_map(&p1.tmap_a, x_perm, 2, H, total_rows);
  if (rc) return rc;
  rc = make_map(&p1.tmap_b, w13_bank, 3, static_cast<uint64_t>(bank_rows) * (2 * I / 128) * (H / BK), 0);
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
  p1.up_tile = I / 128;
  p1.out_ld = I;
  p1.bank_rows = static_cast<int32_t>(bank_rows);
  p1.w_ntiles = 2 * I / 128;
  rc = launch_umma(p1, grid, s, "lm_moe_mlp_prefill: gate_up");
  if (rc) return rc;

  UmmaParams p2 = p1;
  rc = make_map(&p2.tmap_a, act, 2, I, total_rows);
  if (rc) return rc;
  rc = make_map(&p2.tmap_b, w2_bank, 3, static_cast<uint64_t>(bank_rows) * (H / 128) * (I / BK), 0);
  if (rc) return rc;
  p2.out = y_perm;
  p2.k_blocks = I / BK;
  p2.n_tiles = H / BN;
  p2.mode = 1;
  p2.out_ld = H;
  p2.w_ntiles = H / 128;
  return launch_umma(p2, grid, s, "lm_moe_mlp_prefill: down");
}
