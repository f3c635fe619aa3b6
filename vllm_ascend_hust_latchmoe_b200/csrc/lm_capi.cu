// C-ABI glue of liblatchmoe_b200: per-thread error messages, version, and the expert
// staging copy (K10) that moves experts from the pinned host store into slot-bank rows with
// one cudaMemcpyAsync per run of consecutive rows, or from another HBM bank with a copy
// kernel (the copy engine moves device-to-device bytes at a fraction of HBM bandwidth; the
// kernel's CTAs need no shared memory, so they run beside the grouped MLP's CTAs).
#include <string>

#include "lm_common.cuh"

namespace lm {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LM_OK;
  return fail(LM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int launch_status(const char* what) { return check_cuda(cudaGetLastError(), what); }

}  // namespace lm

namespace lm {
namespace {

constexpr int kCopyRowsPerLaunch = 64;
constexpr int64_t kCopyChunk = 64 * 1024;  // bytes per CTA
constexpr int kCopyThreads = 256;

struct CopyRows {
  int32_t src[kCopyRowsPerLaunch];
  int32_t dst[kCopyRowsPerLaunch];
};

// Block (x, y): chunk x of row y; each thread moves 4 x 16 bytes per iteration (four loads in
// flight before the stores). The source is read once (evict-first).
__global__ void __launch_bounds__(kCopyThreads)
    stage_copy_kernel(char* __restrict__ dst, int64_t dst_stride, const char* __restrict__ src,
                      int64_t src_stride, const __grid_constant__ CopyRows rows,
                      int64_t bytes) {
  const int i = blockIdx.y;
  const int64_t off0 = static_cast<int64_t>(blockIdx.x) * kCopyChunk;
  if (off0 >= bytes) return;
  const int64_t len = bytes - off0 < kCopyChunk ? bytes - off0 : kCopyChunk;
  const uint4* s = reinterpret_cast<const uint4*>(src + rows.src[i] * src_stride + off0);
  uint4* d = reinterpret_cast<uint4*>(dst + rows.dst[i] * dst_stride + off0);
  const int64_t n = len / 16;
  for (int64_t c = threadIdx.x; c < n; c += 4 * kCopyThreads) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c + u * kCopyThreads < n) v[u] = __ldcs(s + c + u * kCopyThreads);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c + u * kCopyThreads < n) d[c + u * kCopyThreads] = v[u];
  }
}

// Wave staging driven by a device wave plan: block (x, e) copies chunk x of expert e's row
// into stage row (group - first group of the wave) when the plan put e in wave `wave`
// (expert_to_group[e] in [wave_offsets[wave], wave_offsets[wave + 1])); every other block
// returns at once. Nothing is read on the host, so the staging can be captured.
__global__ void __launch_bounds__(kCopyThreads)
    stage_wave_copy_kernel(char* __restrict__ dst, int64_t dst_stride,
                           const char* __restrict__ src, int64_t src_stride, int64_t bytes,
                           const int32_t* __restrict__ expert_to_group,
                           const int32_t* __restrict__ wave_offsets,
                           const int32_t* __restrict__ num_waves, int wave, int max_rows) {
  if (wave >= *num_waves) return;
  const int e = blockIdx.y;
  const int g = expert_to_group[e];
  const int g0 = wave_offsets[wave], g1 = wave_offsets[wave + 1];
  if (g < g0 || g >= g1 || g - g0 >= max_rows) return;
  const int64_t off0 = static_cast<int64_t>(blockIdx.x) * kCopyChunk;
  if (off0 >= bytes) return;
  const int64_t len = bytes - off0 < kCopyChunk ? bytes - off0 : kCopyChunk;
  const uint4* s = reinterpret_cast<const uint4*>(src + e * src_stride + off0);
  uint4* d = reinterpret_cast<uint4*>(dst + (g - g0) * dst_stride + off0);
  const int64_t n = len / 16;
  for (int64_t c = threadIdx.x; c < n; c += 4 * kCopyThreads) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c + u * kCopyThreads < n) v[u] = __ldcs(s + c + u * kCopyThreads);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c + u * kCopyThreads < n) d[c + u * kCopyThreads] = v[u];
  }
}

}  // namespace
}  // namespace lm

using namespace lm;

extern "C" int lm_abi_version(void) { return LM_ABI_VERSION; }

extern "C" int lm_stage_wave_copy(void* dst, int64_t dst_row_stride, int32_t dst_rows,
                                  const void* src, int64_t src_row_stride, int32_t num_experts,
                                  int64_t bytes_per_expert, const int32_t* expert_to_group,
                                  const int32_t* wave_offsets, const int32_t* num_waves,
                                  int32_t wave, void* stream) {
  if (num_experts <= 0 || num_experts > 65535 || dst_rows <= 0 || wave < 0 ||
      bytes_per_expert <= 0 || dst_row_stride < bytes_per_expert ||
      src_row_stride < bytes_per_expert)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_stage_wave_copy: bad sizes");
  if (dst == nullptr || src == nullptr || expert_to_group == nullptr ||
      wave_offsets == nullptr || num_waves == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_stage_wave_copy: null pointer");
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
        static_cast<uintptr_t>(dst_row_stride) | static_cast<uintptr_t>(src_row_stride) |
        static_cast<uintptr_t>(bytes_per_expert)) & 15) != 0)
    return fail(LM_ERR_INVALID_ARGUMENT,
                "lm_stage_wave_copy: bases, strides and size must be multiples of 16 bytes");
  const dim3 grid(static_cast<unsigned>((bytes_per_expert + kCopyChunk - 1) / kCopyChunk),
                  static_cast<unsigned>(num_experts));
  stage_wave_copy_kernel<<<grid, kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<char*>(dst), dst_row_stride, static_cast<const char*>(src), src_row_stride,
      bytes_per_expert, expert_to_group, wave_offsets, num_waves, wave, dst_rows);
  return launch_status("lm_stage_wave_copy");
}

extern "C" const char* lm_last_error(void) { return g_last_error.c_str(); }

extern "C" int lm_stage_copy(void* dst, int64_t dst_row_stride, const void* src,
                             int64_t src_row_stride, const int32_t* src_rows_host,
                             const int32_t* dst_rows_host, int32_t n, int64_t bytes_per_expert,
                             int32_t kind, void* stream) {
  if (n < 0 || bytes_per_expert <= 0 || dst_row_stride < bytes_per_expert ||
      src_row_stride < bytes_per_expert)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_stage_copy: bad sizes or strides");
  if (kind != LM_COPY_H2D && kind != LM_COPY_D2D)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_stage_copy: kind must be H2D or D2D");
  if (n == 0) return 0;
  if (dst == nullptr || src == nullptr || src_rows_host == nullptr || dst_rows_host == nullptr)
    return fail(LM_ERR_INVALID_ARGUMENT, "lm_stage_copy: null pointer");
  for (int i = 0; i < n; ++i)
    if (src_rows_host[i] < 0 || dst_rows_host[i] < 0)
      return fail(LM_ERR_INVALID_ARGUMENT, "lm_stage_copy: negative row index");
  const cudaMemcpyKind ck = kind == LM_COPY_H2D ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kind == LM_COPY_D2D &&
      ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
        static_cast<uintptr_t>(dst_row_stride) | static_cast<uintptr_t>(src_row_stride) |
        static_cast<uintptr_t>(bytes_per_expert)) & 15) == 0) {
    // device to device: one copy kernel per 64 rows
    int launches = 0;
    for (int i0 = 0; i0 < n; i0 += kCopyRowsPerLaunch) {
      const int m = n - i0 < kCopyRowsPerLaunch ? n - i0 : kCopyRowsPerLaunch;
      CopyRows rows{};
      for (int i = 0; i < m; ++i) {
        rows.src[i] = src_rows_host[i0 + i];
        rows.dst[i] = dst_rows_host[i0 + i];
      }
      const dim3 grid(static_cast<unsigned>((bytes_per_expert + kCopyChunk - 1) / kCopyChunk),
                      static_cast<unsigned>(m));
      stage_copy_kernel<<<grid, kCopyThreads, 0, s>>>(static_cast<char*>(dst), dst_row_stride,
                                                      static_cast<const char*>(src),
                                                      src_row_stride, rows, bytes_per_expert);
      const int rc = launch_status("lm_stage_copy: copy kernel");
      if (rc) return rc;
      ++launches;
    }
    return launches;
  }
  // A run may be merged into one copy only when both sides are densely packed
  // (stride == bytes) and both row sequences advance by one.
  const bool dense = dst_row_stride == bytes_per_expert && src_row_stride == bytes_per_expert;
  int copies = 0;
  int i = 0;
  while (i < n) {
    int j = i + 1;
    if (dense)
      while (j < n && src_rows_host[j] == src_rows_host[j - 1] + 1 &&
             dst_rows_host[j] == dst_rows_host[j - 1] + 1)
        ++j;
    const int run = j - i;
    char* d = static_cast<char*>(dst) + static_cast<int64_t>(dst_rows_host[i]) * dst_row_stride;
    const char* sp =
        static_cast<const char*>(src) + static_cast<int64_t>(src_rows_host[i]) * src_row_stride;
    const int rc = check_cuda(cudaMemcpyAsync(d, sp, bytes_per_expert * run, ck, s),
                              "lm_stage_copy: cudaMemcpyAsync");
    if (rc) return rc;
    ++copies;
    i = j;
  }
  return copies;
}
