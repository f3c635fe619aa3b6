// C-ABI glue of liblatchmoe_b200: per-thread error messages, version, and the expert
// staging copy (K10) that moves experts from the pinned host store (or another HBM bank)
// into slot-bank rows with one cudaMemcpyAsync per run of consecutive rows.
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

using namespace lm;

extern "C" int lm_abi_version(void) { return LM_ABI_VERSION; }

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
