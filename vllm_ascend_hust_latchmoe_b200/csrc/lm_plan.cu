// Device-side canonical wave planner (one CTA): the capacity-bounded wave plan of the
// multi-wave executor computed from the device histogram, so a layer whose experts already
// have an HBM copy needs no device->host round trip to decide its waves.
//
// Plan (identical to the host planner): active experts sorted by (-count, id); ceil(U/S)
// waves; each expert joins the least-loaded wave that still has room (lowest wave index on
// a load tie); members of a wave are ordered by expert id. Groups are numbered wave by
// wave, so the rows of wave w are contiguous after lm_build_groups.
#include "lm_common.cuh"

namespace lm {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxExperts = 1024;

__global__ void __launch_bounds__(kPlanThreads)
    plan_waves_kernel(const int32_t* __restrict__ counts, int num_experts, int num_slots,
                      int bank_row_mode, int32_t* __restrict__ expert_to_group,
                      int32_t* __restrict__ group_bank_row, int32_t* __restrict__ wave_offsets,
                      int32_t* __restrict__ num_waves_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long s_key[kPlanMaxExperts];
  __shared__ int32_t s_wave[kPlanMaxExperts];
  __shared__ long long s_load[kPlanMaxExperts];
  __shared__ int32_t s_size[kPlanMaxExperts];
  __shared__ int32_t s_wave_base[kPlanMaxExperts + 1];
  __shared__ int32_t s_active;
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  int n = 32;  // sort length: next power of two >= num_experts
  while (n < num_experts) n <<= 1;

  // 1) sort keys: active experts by (-count, id); inactive ones sort last.
  for (int e = tid; e < n; e += nthr) {
    unsigned long long key = ~0ull;
    if (e < num_experts) {
      const int c = counts[e];
      if (c > 0)
        key = (static_cast<unsigned long long>(0x7fffffffu - static_cast<unsigned>(c)) << 32) |
              static_cast<unsigned>(e);
    }
    s_key[e] = key;
    s_wave[e] = -1;
  }
  if (tid == 0) s_active = 0;
  __syncthreads();
  int mine = 0;
  for (int e = tid; e < num_experts; e += nthr) mine += counts[e] > 0 ? 1 : 0;
  if (mine) atomicAdd(&s_active, mine);
  // bitonic sort of n keys, ascending
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      __syncthreads();
      for (int i = tid; i < n; i += nthr) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = s_key[i], b = s_key[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            s_key[i] = b;
            s_key[ixj] = a;
          }
        }
      }
    }
  }
  __syncthreads();
  const int U = s_active;
  const int nb = U > 0 ? (U + num_slots - 1) / num_slots : 0;

  // 2) greedy packing by one warp: arg-min load over waves with room, lowest index on ties.
  //    The waves have room for every active expert (nb * num_slots >= U), so a wave with
  //    room always exists.
  if (tid < 32) {
    if (nb <= 32) {
      // Lane w holds wave w: one min-reduction and one ballot per expert. The loads fit
      // 32 bits (they sum to at most the pair count).
      unsigned load = 0;
      int size = 0;
      unsigned long long key = U > 0 ? s_key[0] : 0;
      for (int i = 0; i < U; ++i) {
        const unsigned long long next = i + 1 < U ? s_key[i + 1] : 0;
        const int e = static_cast<int>(key & 0xffffffffu);
        const unsigned c = 0x7fffffffu - static_cast<unsigned>(key >> 32);
        const bool room = tid < nb && size < num_slots;
        const unsigned m = __reduce_min_sync(0xffffffffu, room ? load : 0xffffffffu);
        const unsigned hit = __ballot_sync(0xffffffffu, room && load == m);
        const int bi = __ffs(hit) - 1;
        if (tid == bi) {
          load += c;
          size += 1;
        }
        if (tid == 0) s_wave[e] = bi;
        key = next;
      }
      if (tid < nb) s_size[tid] = size;
    } else {
      for (int w = tid; w < nb; w += 32) {
        s_load[w] = 0;
        s_size[w] = 0;
      }
      __syncwarp();
      for (int i = 0; i < U; ++i) {
        const unsigned long long key = s_key[i];
        const int e = static_cast<int>(key & 0xffffffffu);
        const long long c =
            static_cast<long long>(0x7fffffffu - static_cast<unsigned>(key >> 32));
        long long best = 0x7fffffffffffffffll;
        int bi = 0x7fffffff;
        for (int w = tid; w < nb; w += 32) {
          if (s_size[w] < num_slots && (s_load[w] < best || (s_load[w] == best && w < bi))) {
            best = s_load[w];
            bi = w;
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
        if (tid == 0) {
          s_wave[e] = bi;
          s_load[bi] += c;
          s_size[bi] += 1;
        }
        __syncwarp();
      }
    }
    __syncwarp();
    if (tid == 0) {
      s_wave_base[0] = 0;
      for (int w = 0; w < nb; ++w) s_wave_base[w + 1] = s_wave_base[w] + s_size[w];
    }
  }
  __syncthreads();

  // 3) group index = wave base + rank by expert id inside the wave.
  for (int e = tid; e < num_experts; e += nthr) {
    const int w = s_wave[e];
    int g = -1;
    if (w >= 0) {
      int rank = 0;
      for (int e2 = 0; e2 < e; ++e2) rank += (s_wave[e2] == w) ? 1 : 0;
      g = s_wave_base[w] + rank;
      group_bank_row[g] = bank_row_mode == 0 ? e : rank;
    }
    expert_to_group[e] = g;
  }
  for (int w = tid; w <= nb; w += nthr) wave_offsets[w] = s_wave_base[w];
  if (tid == 0) *num_waves_out = nb;
}

}  // namespace
}  // namespace lm

using namespace lm;

extern "C" int lm_plan_waves(const int32_t* counts, int32_t num_experts, int32_t num_slots,
                             int32_t bank_row_mode, int32_t* expert_to_group,
                             int32_t* group_bank_row, int32_t* wave_offsets,
                             int32_t* num_waves, void* stream) {
  if (num_experts <= 0 || num_experts > kPlanMaxExperts || num_slots <= 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_plan_waves: need 0 < num_experts <= 1024 and num_slots > 0");
  if (bank_row_mode != 0 && bank_row_mode != 1)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_plan_waves: bank_row_mode must be 0 or 1");
  if (counts == nullptr || expert_to_group == nullptr || group_bank_row == nullptr ||
      wave_offsets == nullptr || num_waves == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_plan_waves: null pointer");
  int threads = 32;  // one thread per sort key, at least one warp
  while (threads < num_experts) threads <<= 1;
  const cudaError_t e = launch_dependent(
      plan_waves_kernel, dim3(1), dim3(threads), 0, static_cast<cudaStream_t>(stream), counts,
      num_experts, num_slots, bank_row_mode, expert_to_group, group_bank_row, wave_offsets,
      num_waves);
  if (e != cudaSuccess) return check_cuda(e, "lm_plan_waves");
  return launch_status("lm_plan_waves");
}
