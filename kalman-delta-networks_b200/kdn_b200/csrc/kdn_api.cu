// Host-side error state, version and the packed-batch plan of the kdn_b200
// C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <vector>

#include "kdn_common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

namespace kdn {

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return set_error(KDN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  return KDN_OK;
}

}  // namespace kdn

extern "C" {

int kdn_version(void) { return 102; }

const char* kdn_last_error(void) { return g_last_error; }

int64_t kdn_varlen_table_len(int64_t num_seqs, int64_t num_chunks) {
  return num_seqs > 0 && num_chunks >= num_seqs ? 3 * num_seqs + 2 + num_chunks : 0;
}

int kdn_varlen_plan(const int64_t* cu_seqlens, int64_t num_seqs, int32_t* table, int64_t table_len,
                    int64_t* num_chunks) {
  using kdn::kVarlenChunk;
  if (!cu_seqlens || num_seqs <= 0 || !num_chunks)
    return kdn::set_error(KDN_ERR_INVALID, "kdn_varlen_plan: cu_seqlens, num_seqs > 0 and num_chunks required");
  if (cu_seqlens[0] != 0) return kdn::set_error(KDN_ERR_INVALID, "kdn_varlen_plan: cu_seqlens must start at 0");
  int64_t nc = 0;
  for (int64_t i = 0; i < num_seqs; ++i) {
    const int64_t len = cu_seqlens[i + 1] - cu_seqlens[i];
    if (len <= 0) return kdn::set_error(KDN_ERR_INVALID, "kdn_varlen_plan: cu_seqlens must increase strictly");
    nc += (len + kVarlenChunk - 1) / kVarlenChunk;
  }
  if (cu_seqlens[num_seqs] > INT32_MAX || nc > INT32_MAX / kVarlenChunk)
    return kdn::set_error(KDN_ERR_INVALID, "kdn_varlen_plan: size too large");
  *num_chunks = nc;
  if (!table) return KDN_OK;
  if (table_len < kdn_varlen_table_len(num_seqs, nc))
    return kdn::set_error(KDN_ERR_INVALID, "kdn_varlen_plan: table needs %lld entries",
                          (long long)kdn_varlen_table_len(num_seqs, nc));
  int32_t* tok = table;
  int32_t* chunk = tok + (num_seqs + 1);
  int32_t* order = chunk + (num_seqs + 1);
  int32_t* seq = order + num_seqs;
  chunk[0] = 0;
  for (int64_t i = 0; i <= num_seqs; ++i) tok[i] = (int32_t)cu_seqlens[i];
  for (int64_t i = 0; i < num_seqs; ++i) {
    const int32_t n = (int32_t)((cu_seqlens[i + 1] - cu_seqlens[i] + kVarlenChunk - 1) / kVarlenChunk);
    chunk[i + 1] = chunk[i] + n;
    for (int32_t c = chunk[i]; c < chunk[i + 1]; ++c) seq[c] = (int32_t)i;
  }
  std::vector<int32_t> idx((size_t)num_seqs);
  for (int64_t i = 0; i < num_seqs; ++i) idx[(size_t)i] = (int32_t)i;
  std::stable_sort(idx.begin(), idx.end(), [&](int32_t a, int32_t b) {
    return cu_seqlens[a + 1] - cu_seqlens[a] > cu_seqlens[b + 1] - cu_seqlens[b];
  });
  for (int64_t i = 0; i < num_seqs; ++i) order[i] = idx[(size_t)i];
  return KDN_OK;
}

}  // extern "C"
