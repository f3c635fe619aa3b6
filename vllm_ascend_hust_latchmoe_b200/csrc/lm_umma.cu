// Prefill path of the grouped expert MLP on the 5th-generation tensor cores (tcgen05).
//
// Persistent kernels run both GEMMs of the expert MLP (selected by `mode`):
//   mode 0 (gate_up): act[r, n0:n0+128] = silu(X_r . W13[n0:n0+128]) * (X_r . W13[I+n0:...])
//                     MMA N = 256 = 128 gate rows + the 128 matching up rows, so the fused
//                     SiLU*mul epilogue has both halves of every output column in TMEM.
//   mode 1 (down):    y[r, n0:n0+256] = act_r . W2[n0:n0+256]
//
// Measured on B200, these facts shape the kernels:
//  * a tcgen05.mma of K = 16 costs about the same time for any N up to 256, and with
//    cta_group::2 each SM supplies only half of the instruction's N rows;
//  * one thread issues TMA loads at a limited rate, and each pipeline stage hand-off has a
//    fixed cost, whatever the bytes moved.
// So the groups of a call are split by size. Groups of more than LIGHT_MAX_ROWS rows
// ("heavy": each weight tile serves many rows; tensor-bound) run on 2-SM tiles of
// 256 x 256 (umma_grouped_kernel_2sm, cta_group::2; per K block each SM loads 32 KiB for
// 128 x 256 MMA work). The other groups ("light": bound by streaming their weights) run on
// single-SM tiles of 128 x 256 (umma_grouped_kernel), where one instruction consumes 256
// weight rows per SM and only the group's rows of A are loaded. The two kinds are launched
// on two streams, both with one CTA per SM; each launch derives the same split of the SMs
// from group_offsets (in proportion to the estimated SM time of each kind), and CTAs beyond
// their launch's share leave at once, handing their SMs to the other launch. With
// LM_UMMA_CTA_PAIR=1 every group runs on the single-SM kernel over all SMs.
//
// Loads of a stage are issued by several lanes at once (one TMA load each), and two producer
// warps take the stages in turn. Warp roles (224 threads): warps 0 and 6 issue TMA loads into
// the smem ring, warp 1 issues tcgen05.mma into one of two TMEM accumulators (2 x 256 fp32
// columns = all 512 columns), warps 2-5 drain the other accumulator (tcgen05.ld -> epilogue
// -> global stores), so the epilogue of tile i overlaps the MMAs of tile i+1. The tile list
// (group, m-tile, n-tile; n fastest) is derived on the device from group_offsets, so the
// launches are independent of the routing.
// No TMA load uses cluster multicast; every operand is this GPU's own memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "lm_common.cuh"
#include "lm_tmap.cuh"

namespace lm {
namespace {

constexpr int BM = 128;   // rows per CTA (TMEM lanes)
constexpr int BN = 256;   // MMA N (mode 0: 128 gate + 128 up rows; mode 1: 256 outputs)
constexpr int BK = 64;    // one 128-byte swizzle row of bf16
constexpr int KB_BYTES = BM * BK * 2;  // one 128-row x 64 K block, 16 KiB
constexpr int TMEM_COLS = 512;
constexpr int MAX_G = 256;
constexpr int NUM_THREADS = 224;  // warps 0, 6: TMA; 1: MMA; 2-5: epilogue
constexpr int NUM_PRODUCERS = 2;
constexpr int MAX_STAGES = 4;
constexpr int LIGHT_MAX_ROWS = 128;  // larger groups run on 2-SM tiles
// Single-SM tiles prefetch their weight tiles into L2 this many K blocks ahead of the loads
// (even): light tiles stream weights from DRAM, and the prefetches keep more bytes in
// flight than the shared-memory ring can hold.
constexpr int PREFETCH_KB = 8;

enum : int32_t { ROLE_HEAVY = 0, ROLE_LIGHT = 1, ROLE_ALL = 2 };

// PAIR = 1: one CTA owns a 128-row tile; a stage is one K block: its rows (16 KiB at most)
// and the 256 weight rows (both 128-row tiles, 32 KiB).
// PAIR = 2: a cluster of two CTAs owns a 256-row tile (M = 256, cta_group::2); a stage is two
// K blocks: each CTA's 128 rows (32 KiB) and its one weight tile (32 KiB); the leader issues
// the MMAs.
template <int PAIR>
struct Cfg {
  static constexpr int KB_STAGE = PAIR == 1 ? 1 : 2;
  static constexpr int A_BYTES = KB_STAGE * KB_BYTES;
  static constexpr int B_BYTES = KB_STAGE * KB_BYTES * (PAIR == 1 ? 2 : 1);
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR == 1 ? 4 : 3;
  static constexpr int UNIT_ROWS = BM * PAIR;
};

struct SmemCtl {
  uint4 xpose[4][128];     // per epilogue warp: 32 rows x 64 B, for coalesced output stores
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int units_other;         // unit-tiles of the other kind (heavy / light split)
  int prefix[MAX_G + 1];   // unit-tiles of this launch's groups before group i
  int row0[MAX_G];
  int nrows[MAX_G];
  int bank[MAX_G];
};

template <int PAIR>
constexpr int smem_bytes() {
  return 1024 + Cfg<PAIR>::STAGES * Cfg<PAIR>::STAGE_BYTES + static_cast<int>(sizeof(SmemCtl));
}

struct UmmaParams {
  CUtensorMap tmap_a[4];  // A rows [R, K] bf16, boxes {64, 16 / 32 / 64 / 128}
  CUtensorMap tmap_w2;    // weight tiles [tiles][128][64], box {64, 128, 2}: K blocks kb, kb+1
  CUtensorMap tmap_w1;    // the same tiles, box {64, 128, 1}
  const int32_t* group_offsets;
  const int32_t* group_bank_row;
  uint16_t* out;
  uint16_t* const* row_ptr;  // mode 1: output row r goes to row_ptr[r] (may be a peer's memory)
  // device-side group range: the groups of wave `wave` of a device wave plan,
  // [wave_offsets[wave], wave_offsets[wave + 1]), none when wave >= *num_waves
  const int32_t* wave_offsets;
  const int32_t* num_waves;
  int32_t wave;
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
  int32_t role;      // ROLE_HEAVY (2-SM kernel), ROLE_LIGHT or ROLE_ALL (1-SM kernel)
  int32_t split_sms;         // SMs shared by the heavy and the light launch
  int32_t heavy_tile_cost;   // estimated SM time of a heavy tile, per SM of the pair
  int32_t light_tile_cost;   // estimated SM time of a light tile
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

// Position t of the tile list -> (group, unit-tile, n-tile).
__device__ __forceinline__ TileCoord decode_tile(const SmemCtl& c, int t, int n_tiles, int G,
                                                 int unit) {
  TileCoord tc;
  const int mg = t / n_tiles;
  tc.nt = t - mg * n_tiles;
  const int g = find_group(c.prefix, mg, G);
  const int ml = mg - c.prefix[g];
  tc.g = g;
  tc.row0 = c.row0[g] + ml * unit;
  const int rem = c.nrows[g] - ml * unit;
  tc.valid = rem < unit ? rem : unit;
  return tc;
}

// Rows of A loaded for a single-SM tile: the tile's rows rounded up to 16 / 32 / 64 / 128
// (the rest of the 128-row operand is left as it is; those accumulator rows are not stored).
__device__ __forceinline__ int a_box_index(int valid) {
  return valid <= 16 ? 0 : valid <= 32 ? 1 : valid <= 64 ? 2 : 3;
}

// One epilogue warp's 32-row x 32-column bf16 chunk (lane = row, 64 B each in `packed`) to
// global memory. A lane-per-row store would touch 32 rows per instruction; instead the rows
// pass through a 2 KiB shared buffer (16-byte chunk c of row r at r * 64 + ((c ^ (r >> 1 & 3))
// * 16), conflict-free both ways) and each store instruction writes 8 rows x 64 contiguous
// bytes. Rows at or past `valid_rows` (of this warp's 32) are not written.
__device__ __forceinline__ void store_chunk_coalesced(uint4* xbuf, uint16_t* out0, int64_t ld,
                                                      int valid_rows,
                                                      const uint32_t (&packed)[16]) {
  const int lane = threadIdx.x & 31;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    xbuf[lane * 4 + (c ^ sw)] =
        make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
  __syncwarp();
  const int cc = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = 8 * i + (lane >> 2);
    const uint4 v = xbuf[row * 4 + (cc ^ ((row >> 1) & 3))];
    if (row < valid_rows) *reinterpret_cast<uint4*>(out0 + row * ld + cc * 8) = v;
  }
  __syncwarp();
}

// The same chunk stored through per-row pointers (lane_row = the pointer of this warp's row
// `lane`, which may address another GPU's memory): each store instruction still writes 8 rows
// x 64 contiguous bytes.
__device__ __forceinline__ void store_chunk_rows(uint4* xbuf, uint16_t* lane_row, int col,
                                                 int valid_rows, const uint32_t (&packed)[16]) {
  const int lane = threadIdx.x & 31;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    xbuf[lane * 4 + (c ^ sw)] =
        make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
  __syncwarp();
  const int cc = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = 8 * i + (lane >> 2);
    const uint4 v = xbuf[row * 4 + (cc ^ ((row >> 1) & 3))];
    uint16_t* rp = reinterpret_cast<uint16_t*>(
        __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(lane_row), row));
    if (row < valid_rows) *reinterpret_cast<uint4*>(rp + col + cc * 8) = v;
  }
  __syncwarp();
}

// Clusters of a launch that take tiles. For the heavy / light pair of launches both compute
// the same split of split_sms SMs from the same inputs.
__device__ __forceinline__ int active_clusters(const UmmaParams& p, int own_units,
                                               int other_units, int num_clusters) {
  if (p.role == ROLE_ALL) return num_clusters;
  const long long ht =
      static_cast<long long>(p.role == ROLE_HEAVY ? own_units : other_units) * p.n_tiles;
  const long long lt =
      static_cast<long long>(p.role == ROLE_LIGHT ? own_units : other_units) * p.n_tiles;
  const int sms = p.split_sms;
  const long long wh = ht * 2 * p.heavy_tile_cost, wl = lt * p.light_tile_cost;
  long long heavy_sms = wh + wl > 0 ? (sms * wh + (wh + wl) / 2) / (wh + wl) : 0;
  heavy_sms &= ~1ll;
  if (heavy_sms > 2 * ht) heavy_sms = 2 * ht;                       // no more pairs than tiles
  if (sms - heavy_sms > lt) heavy_sms = (sms - lt + 1) & ~1ll;      // no more SMs than tiles
  if (heavy_sms > 2 * ht) heavy_sms = 2 * ht;
  if (ht > 0 && heavy_sms < 2) heavy_sms = 2;
  if (lt > 0 && heavy_sms > ((sms - 1) & ~1)) heavy_sms = (sms - 1) & ~1;
  long long active = p.role == ROLE_HEAVY ? heavy_sms / 2 : sms - heavy_sms;
  if (active > num_clusters) active = num_clusters;
  return static_cast<int>(active);
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
  int G = p.num_groups;
  int gbeg = p.group_begin;
  if (p.wave_offsets != nullptr) {
    G = 0;
    if (p.wave < *p.num_waves) {
      gbeg = p.wave_offsets[p.wave];
      const int n = p.wave_offsets[p.wave + 1] - gbeg;
      if (n > MAX_G) {
        if (threadIdx.x == 0 && p.role != ROLE_LIGHT) record_error(p.err_word, LM_DEVERR_BAD_GROUP);
      } else if (n > 0 && gbeg >= 0) {
        G = n;
      }
    }
  }
  const uint32_t rank = PAIR == 2 ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x / PAIR;
  const int num_clusters = gridDim.x / PAIR;
  const int ksteps = p.k_blocks / C::KB_STAGE;

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
  for (int i = threadIdx.x; i < G; i += NUM_THREADS) {
    const int g = gbeg + i;
    const int r0 = p.group_offsets[g];
    int n = p.group_offsets[g + 1] - r0;
    int bank = p.group_bank_row[g];
    if (n > 0 && (bank < 0 || bank >= p.bank_rows)) {
      if (p.role != ROLE_LIGHT) record_error(p.err_word, LM_DEVERR_BAD_GROUP);
      n = 0;
      bank = 0;
    }
    c.row0[i] = r0;
    c.nrows[i] = n > 0 ? n : 0;
    c.bank[i] = bank;
  }
  __syncthreads();
  if (warp == 0) {
    // prefix of unit-tiles over this launch's groups; unit-tiles of the other kind
    int carry = 0, other = 0;
    for (int base = 0; base < G; base += 32) {
      const int i = base + lane;
      const int n = (i < G) ? c.nrows[i] : 0;
      const bool heavy = n > LIGHT_MAX_ROWS;
      const bool mine =
          n > 0 && (p.role == ROLE_ALL || (p.role == ROLE_HEAVY) == heavy);
      int v = mine ? (n + C::UNIT_ROWS - 1) / C::UNIT_ROWS : 0;
      if (!mine && n > 0 && p.role != ROLE_ALL) other += heavy ? (n + 2 * BM - 1) / (2 * BM) : 1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (i < G) c.prefix[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) other += __shfl_xor_sync(0xffffffffu, other, o);
    if (lane == 0) {
      c.prefix[0] = 0;
      c.units_other = other;
    }
  }
  __syncthreads();

  const int total_tiles = c.prefix[G] * p.n_tiles;
  const int active = active_clusters(p, c.prefix[G], c.units_other, num_clusters);
  // Both CTAs of a cluster reach the same decision; an idle CTA leaves before taking TMEM,
  // so its SM goes to the other launch right away.
  if (cluster_id >= active || total_tiles == 0) return;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 4; ++i) tma_prefetch_desc(&p.tmap_a[i]);
    tma_prefetch_desc(&p.tmap_w2);
    tma_prefetch_desc(&p.tmap_w1);
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
  tc_fence_before();
  __syncthreads();
  if (PAIR == 2) cluster_sync_all();  // peer barriers initialised, both TMEM halves allocated
  tc_fence_after();
  const uint32_t tmem_base = c.tmem_base;
  volatile int* abort_flag = &c.abort_flag;

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------------ TMA producers
    // Producer pw issues the pipeline steps seq with seq % 2 == pw (a step = one stage of one
    // tile); lane i of the warp issues the i-th load of the step.
    const int pw = warp == 0 ? 0 : 1;
    int seq = 0;
    bool ok = true;
    for (int t = cluster_id; t < total_tiles && ok; t += active) {
      const TileCoord tc = decode_tile(c, t, p.n_tiles, G, C::UNIT_ROWS);
      const int ebase = c.bank[tc.g] * p.w_ntiles;
      // weight tiles of the n-tile: gate / up (mode 0) or two consecutive W2 tiles (mode 1)
      const int wt0 = ebase + (p.mode == 0 ? tc.nt : 2 * tc.nt);
      const int wt1 = ebase + (p.mode == 0 ? p.up_tile + tc.nt : 2 * tc.nt + 1);
      const int abox = PAIR == 1 ? a_box_index(tc.valid) : 3;
      const uint32_t bytes = PAIR == 2 ? C::STAGE_BYTES : (16u << abox) * BK * 2 + C::B_BYTES;
      for (int ks = 0; ks < ksteps; ++ks, ++seq) {
        if (seq % NUM_PRODUCERS != pw) continue;
        const int stage = seq % C::STAGES;
        const uint32_t phase = static_cast<uint32_t>(seq / C::STAGES) & 1u;
        bool got = true;
        if (lane == 0) got = mbar_wait_bounded(&c.empty[stage], phase ^ 1u, p.err_word, abort_flag);
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        if (!got) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * C::STAGE_BYTES;
        uint8_t* sb = sa + C::A_BYTES;
        const int kb = ks * C::KB_STAGE;
        if (PAIR == 2) {
          // Both CTAs' bytes complete on the leader's barrier; only the leader arrives.
          const uint32_t full_leader = mapa_shared(smem_u32(&c.full[stage]), 0);
          if (lane == 0 && leader) mbar_arrive_expect_tx(&c.full[stage], 2 * bytes);
          __syncwarp();
          if (lane < 2) {
            tma_load_2d_pair(sa + lane * KB_BYTES, &p.tmap_a[3], full_leader, (kb + lane) * BK,
                             tc.row0 + static_cast<int>(rank) * BM);
          } else if (lane == 2) {
            const int wt = rank == 0 ? wt0 : wt1;
            tma_load_3d_pair(sb, &p.tmap_w2, full_leader, 0, 0, wt * p.k_blocks + kb);
          }
        } else {
          if (lane == 0) mbar_arrive_expect_tx(&c.full[stage], bytes);
          __syncwarp();
          if (lane == 0) {
            tma_load_2d(sa, &p.tmap_a[abox], &c.full[stage], kb * BK, tc.row0);
          } else if (lane <= 2) {
            const int wt = lane == 1 ? wt0 : wt1;
            tma_load_3d(sb + (lane - 1) * KB_BYTES, &p.tmap_w1, &c.full[stage], 0, 0,
                        wt * p.k_blocks + kb);
          } else if (lane <= 4 && p.role == ROLE_LIGHT) {
            // weight tiles of K blocks (kb + PREFETCH_KB, +1), two per prefetch; at the
            // tile's first step also the K blocks before that
            const int wt = lane == 3 ? wt0 : wt1;
            const int kp = kb + PREFETCH_KB;
            if ((kp & 1) == 0 && kp < p.k_blocks)
              tma_prefetch_l2_3d(&p.tmap_w2, 0, 0, wt * p.k_blocks + kp);
            if (ks == 0)
              for (int k2 = 2; k2 < PREFETCH_KB && k2 < p.k_blocks; k2 += 2)
                tma_prefetch_l2_3d(&p.tmap_w2, 0, 0, wt * p.k_blocks + k2);
          }
        }
        __syncwarp();
      }
    }
    // Producer 0 waits until the MMAs released every stage of every step this CTA issued
    // (by either producer), so no TMA write or commit arrival into this CTA's shared memory
    // is still in flight at exit.
    if (warp == 0 && lane == 0) {
      int total = 0;
      for (int t = cluster_id; t < total_tiles; t += active) total += ksteps;
      for (int s = 0; s < C::STAGES && s < total; ++s) {
        const int last = s + ((total - 1 - s) / C::STAGES) * C::STAGES;
        const uint32_t par = static_cast<uint32_t>(last / C::STAGES) & 1u;
        const long long t0 = clock64();
        while (!mbar_try_wait(&c.empty[s], par) && clock64() - t0 < LM_SPIN_LIMIT_CYCLES) {
          if (*abort_flag && clock64() - t0 > 200000) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(BM * PAIR, BN);
      int seq = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster_id; t < total_tiles && ok; t += active) {
        if (!mbar_wait_bounded(&c.tempty[acc], acc_phase ^ 1u, p.err_word, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int ks = 0; ks < ksteps; ++ks, ++seq) {
          const int stage = seq % C::STAGES;
          const uint32_t phase = static_cast<uint32_t>(seq / C::STAGES) & 1u;
          if (!mbar_wait_bounded(&c.full[stage], phase, p.err_word, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int j = 0; j < C::KB_STAGE; ++j) {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad = sdesc_k_sw128(a_addr + j * KB_BYTES + kk * 32);
              const uint64_t bd = sdesc_k_sw128(b_addr + j * KB_BYTES + kk * 32);
              const uint32_t accum = (ks | j | kk) != 0 ? 1u : 0u;
              if (PAIR == 2)
                umma_bf16_pair(d_tmem, ad, bd, idesc, accum);
              else
                umma_bf16(d_tmem, ad, bd, idesc, accum);
            }
          }
          if (PAIR == 2)
            umma_commit_pair(&c.empty[stage], 0x3);
          else
            umma_commit(&c.empty[stage]);
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
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&c.tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&c.tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster_id; t < total_tiles; t += active) {
      const TileCoord tc = decode_tile(c, t, p.n_tiles, G, C::UNIT_ROWS);
      if (!mbar_wait_bounded(&c.tfull[acc], acc_phase, p.err_word, abort_flag)) break;
      tc_fence_after();
      const int my_valid = tc.valid - static_cast<int>(rank) * BM;
      const int warp_rows = my_valid - quad * 32;  // rows of this warp's 32 in the tile
      uint16_t* out_warp = p.out + static_cast<int64_t>(tc.row0 + static_cast<int>(rank) * BM +
                                                        quad * 32) * p.out_ld;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      // Warps whose 32 lanes are all past the tile's rows only release the accumulator.
      if (quad * 32 < my_valid) {
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
            store_chunk_coalesced(c.xpose[quad], out_warp + tc.nt * 128 + ch * 32, p.out_ld,
                                  warp_rows, packed);
          }
        } else if (p.row_ptr != nullptr) {
          // this lane's row: its output pointer (the rows past the tile's are never stored)
          const int rr = quad * 32 + lane;
          uint16_t* lane_row = rr < my_valid
                                   ? p.row_ptr[tc.row0 + static_cast<int>(rank) * BM + rr]
                                   : nullptr;
#pragma unroll 1
          for (int ch = 0; ch < 8; ++ch) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tbase + ch * 32, v);
            tmem_ld_wait();
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              packed[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            store_chunk_rows(c.xpose[quad], lane_row, tc.nt * BN + ch * 32, warp_rows, packed);
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
            store_chunk_coalesced(c.xpose[quad], out_warp + tc.nt * BN + ch * 32, p.out_ld,
                                  warp_rows, packed);
          }
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
    // stores through row pointers may have gone to other GPUs: order them before anything
    // this thread's stream does next (the exchange's signal follows this kernel)
    if (p.row_ptr != nullptr) __threadfence_system();
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

// Heavy groups on 2-SM tiles beside light groups on single-SM tiles by default;
// LM_UMMA_CTA_PAIR=1 runs every group on the single-SM kernel.
int cta_pair() {
  static int v = [] {
    const char* e = getenv("LM_UMMA_CTA_PAIR");
    return (e != nullptr && e[0] == '1') ? 1 : 2;
  }();
  return v;
}

// Relative SM time of a heavy tile (per SM of its pair) and of a light tile, per GEMM (mode),
// for the split of the SMs between the two launches; measured on the 4096-token
// Qwen3-30B-A3B layer (gate_up 4:5, down 5:5). LM_UMMA_SPLIT_COST="h0:l0:h1:l1" overrides.
void split_costs(int mode, int* heavy, int* light) {
  static int c[4] = {4, 5, 5, 5};
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = getenv("LM_UMMA_SPLIT_COST");
    int v[4] = {0, 0, 0, 0};
    if (e != nullptr && sscanf(e, "%d:%d:%d:%d", &v[0], &v[1], &v[2], &v[3]) == 4 &&
        v[0] > 0 && v[1] > 0 && v[2] > 0 && v[3] > 0)
      for (int i = 0; i < 4; ++i) c[i] = v[i];
  });
  *heavy = c[2 * mode];
  *light = c[2 * mode + 1];
}

// Per-device side stream for the light launches, with the fork / join events. Calls hold the
// mutex from the fork to the join, so the shared events are never re-recorded before the
// waits on them are enqueued.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr;
  cudaEvent_t join = nullptr;
};

std::mutex& side_mutex() {
  static std::mutex mu;
  return mu;
}

int side_stream(SideStream** out) {
  static SideStream per_dev[64];
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "lm_moe_mlp_prefill: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(LM_ERR_UNSUPPORTED, "lm_moe_mlp_prefill: device index >= 64");
  SideStream& ss = per_dev[dev];
  if (ss.stream == nullptr) {
    rc = check_cuda(cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking),
                    "lm_moe_mlp_prefill: side stream");
    if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming),
                             "lm_moe_mlp_prefill: fork event");
    if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming),
                             "lm_moe_mlp_prefill: join event");
    if (rc) return rc;
  }
  *out = &ss;
  return LM_OK;
}

int launch_umma(UmmaParams p, int role, int grid, cudaStream_t s, const char* what) {
  p.role = role;
  if (role == ROLE_HEAVY) {
    umma_grouped_kernel_2sm<<<grid & ~1, NUM_THREADS, smem_bytes<2>(), s>>>(p);
  } else {
    umma_grouped_kernel<<<grid, NUM_THREADS, smem_bytes<1>(), s>>>(p);
  }
  return launch_status(what);
}

// Activation-row maps: boxes of 16 / 32 / 64 / 128 rows over the same rows.
int make_row_maps(CUtensorMap* maps, const void* ptr, uint64_t k, uint64_t rows) {
  for (int i = 0; i < 4; ++i) {
    int rc = make_map(&maps[i], ptr, 2, k, rows, 16 << i);
    if (rc) return rc;
  }
  return LM_OK;
}

}  // namespace
}  // namespace lm

using namespace lm;

namespace {
int prefill_impl(const uint16_t* x_perm, int64_t total_rows, const int32_t* group_offsets,
                 const int32_t* group_bank_row, int32_t group_begin, int32_t group_end,
                 const uint16_t* w13_bank, const uint16_t* w2_bank, int64_t bank_rows,
                 int32_t hidden_size, int32_t intermediate_size, uint16_t* act,
                 uint16_t* y_perm, uint16_t* const* y_rows, int32_t* err_word, void* stream,
                 const int32_t* wave_offsets = nullptr, const int32_t* num_waves = nullptr,
                 int32_t wave = 0) {
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
      w13_bank == nullptr || w2_bank == nullptr || act == nullptr ||
      (y_perm == nullptr) == (y_rows == nullptr))
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
  const uint64_t w13_tiles = static_cast<uint64_t>(bank_rows) * (2 * I / 128) * (H / BK);
  rc = make_row_maps(p1.tmap_a, x_perm, H, total_rows);
  if (!rc) rc = make_map(&p1.tmap_w2, w13_bank, 3, w13_tiles, 0, 128, 2);
  if (!rc) rc = make_map(&p1.tmap_w1, w13_bank, 3, w13_tiles, 0, 128, 1);
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
  p1.split_sms = grid;
  p1.wave_offsets = wave_offsets;
  p1.num_waves = num_waves;
  p1.wave = wave;
  split_costs(0, &p1.heavy_tile_cost, &p1.light_tile_cost);

  UmmaParams p2 = p1;
  const uint64_t w2_tiles = static_cast<uint64_t>(bank_rows) * (H / 128) * (I / BK);
  rc = make_row_maps(p2.tmap_a, act, I, total_rows);
  if (!rc) rc = make_map(&p2.tmap_w2, w2_bank, 3, w2_tiles, 0, 128, 2);
  if (!rc) rc = make_map(&p2.tmap_w1, w2_bank, 3, w2_tiles, 0, 128, 1);
  if (rc) return rc;
  p2.out = y_perm;
  p2.row_ptr = y_rows;
  p2.k_blocks = I / BK;
  p2.n_tiles = H / BN;
  p2.mode = 1;
  p2.out_ld = H;
  p2.w_ntiles = H / 128;
  split_costs(1, &p2.heavy_tile_cost, &p2.light_tile_cost);

  if (cta_pair() == 1) {
    rc = launch_umma(p1, ROLE_ALL, grid, s, "lm_moe_mlp_prefill: gate_up");
    if (!rc) rc = launch_umma(p2, ROLE_ALL, grid, s, "lm_moe_mlp_prefill: down");
    return rc;
  }
  // Heavy groups: the 2-SM launches on the caller's stream. Light groups: the single-SM
  // launches on the side stream, forked after the caller's prior work and joined back before
  // anything the caller enqueues next; the light down GEMM starts as soon as the light
  // gate_up is done, while the heavy gate_up may still run. Each GEMM's pair of launches
  // splits the SMs between them; the CTAs a launch does not need leave at once.
  std::lock_guard<std::mutex> lk(side_mutex());
  SideStream* ss = nullptr;
  rc = side_stream(&ss);
  if (!rc) rc = check_cuda(cudaEventRecord(ss->fork, s), "lm_moe_mlp_prefill: fork");
  if (!rc) rc = check_cuda(cudaStreamWaitEvent(ss->stream, ss->fork, 0), "lm_moe_mlp_prefill: fork wait");
  if (rc) return rc;
  rc = launch_umma(p1, ROLE_HEAVY, grid, s, "lm_moe_mlp_prefill: gate_up (2-SM)");
  if (!rc) rc = launch_umma(p1, ROLE_LIGHT, grid, ss->stream, "lm_moe_mlp_prefill: gate_up (1-SM)");
  if (!rc) rc = launch_umma(p2, ROLE_HEAVY, grid, s, "lm_moe_mlp_prefill: down (2-SM)");
  if (!rc) rc = launch_umma(p2, ROLE_LIGHT, grid, ss->stream, "lm_moe_mlp_prefill: down (1-SM)");
  // Join even after a failed launch, so the caller's stream never runs ahead of the side.
  const int rj = check_cuda(cudaEventRecord(ss->join, ss->stream), "lm_moe_mlp_prefill: join");
  const int rw = rj ? rj : check_cuda(cudaStreamWaitEvent(s, ss->join, 0), "lm_moe_mlp_prefill: join wait");
  return rc ? rc : rw;
}
}  // namespace

extern "C" int lm_moe_mlp_prefill(const uint16_t* x_perm, int64_t total_rows,
                                  const int32_t* group_offsets, const int32_t* group_bank_row,
                                  int32_t group_begin, int32_t group_end,
                                  const uint16_t* w13_bank, const uint16_t* w2_bank,
                                  int64_t bank_rows, int32_t hidden_size,
                                  int32_t intermediate_size, uint16_t* act, uint16_t* y_perm,
                                  int32_t* err_word, void* stream) {
  return prefill_impl(x_perm, total_rows, group_offsets, group_bank_row, group_begin, group_end,
                      w13_bank, w2_bank, bank_rows, hidden_size, intermediate_size, act, y_perm,
                      nullptr, err_word, stream);
}

extern "C" int lm_moe_mlp_prefill_rows(const uint16_t* x_perm, int64_t total_rows,
                                       const int32_t* group_offsets,
                                       const int32_t* group_bank_row, int32_t group_begin,
                                       int32_t group_end, const uint16_t* w13_bank,
                                       const uint16_t* w2_bank, int64_t bank_rows,
                                       int32_t hidden_size, int32_t intermediate_size,
                                       uint16_t* act, uint16_t* const* y_row_ptrs,
                                       int32_t* err_word, void* stream) {
  if (y_row_ptrs == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_prefill_rows: null row pointers");
  return prefill_impl(x_perm, total_rows, group_offsets, group_bank_row, group_begin, group_end,
                      w13_bank, w2_bank, bank_rows, hidden_size, intermediate_size, act, nullptr,
                      y_row_ptrs, err_word, stream);
}

extern "C" int lm_moe_mlp_prefill_wave(const uint16_t* x_perm, int64_t total_rows,
                                       const int32_t* group_offsets,
                                       const int32_t* group_bank_row,
                                       const int32_t* wave_offsets, const int32_t* num_waves,
                                       int32_t wave, const uint16_t* w13_bank,
                                       const uint16_t* w2_bank, int64_t bank_rows,
                                       int32_t hidden_size, int32_t intermediate_size,
                                       uint16_t* act, uint16_t* y_perm, int32_t* err_word,
                                       void* stream) {
  if (wave_offsets == nullptr || num_waves == nullptr || wave < 0)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_moe_mlp_prefill_wave: bad wave arguments");
  // the group range comes from the device plan; [0, 1) only passes the host checks
  return prefill_impl(x_perm, total_rows, group_offsets, group_bank_row, 0, 1, w13_bank,
                      w2_bank, bank_rows, hidden_size, intermediate_size, act, y_perm, nullptr,
                      err_word, stream, wave_offsets, num_waves, wave);
}
