// linattn_sparse_attention_noalloc: the split-KV sparse attention with its scratch
// space in a fixed device array owned by this library instead of a caller buffer.
//
// Some callers cannot allocate device memory where they run attention: a host
// engine that reserves all of HBM for its own pool and forbids side allocations, or
// a latency-critical path that cannot afford cudaMalloc's implicit device
// synchronisation.  This entry point takes the same inputs and outputs as
// linattn_sparse_attention but no workspace: the split-KV partials live in the
// file-scope array below (64 MiB), which every GPU that loads the library holds
// until the process exits.  Calls share it, so calls that overlap on the GPU (two
// streams, or two host threads) race on it; the array keeps the last call's
// contents and every call overwrites what it reads.
#include <cstdio>
#include <mutex>

#include "launchers.cuh"

namespace {

constexpr int64_t kNoAllocScratchBytes = 64ll << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[64] = {};

}  // namespace

extern "C" {

int64_t linattn_sparse_attention_noalloc_limit(void) { return kNoAllocScratchBytes; }

int linattn_sparse_attention_noalloc(const void* q, int32_t q_dtype, int64_t B, int64_t Hq, int64_t Tq,
                                     const int64_t* q_strides, const linattn_kv_t* kv, const linattn_lists_t* lists,
                                     int32_t causal, int64_t offset, float scale, void* out,
                                     const int64_t* out_strides, float* lse_out, int32_t n_splits, int32_t* status,
                                     void* stream) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return linattn::set_error(LINATTN_ECUDA, "sparse_attention_noalloc: no current CUDA device (or index >= 64)");
  void* scratch = nullptr;
  {
    // In host code g_noalloc_scratch names a host-side stand-in, not a device
    // address: resolve the device address once per device, with it current.
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        char msg[256];
        snprintf(msg, sizeof(msg), "sparse_attention_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
        return linattn::set_error(LINATTN_ECUDA, msg);
      }
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  if (kv == nullptr) return linattn::set_error(LINATTN_EINVAL, "sparse_attention_noalloc: kv descriptor is NULL");
  const int64_t need = linattn_sparse_attention_workspace(B, Hq, Tq, kv->head_dim, n_splits);
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg), "sparse_attention_noalloc: needs %lld bytes of scratch, limit is %lld",
             static_cast<long long>(need), static_cast<long long>(kNoAllocScratchBytes));
    return linattn::set_error(LINATTN_EINVAL, msg);
  }
  return linattn_sparse_attention(q, q_dtype, B, Hq, Tq, q_strides, kv, lists, causal, offset, scale, out,
                                  out_strides, lse_out, n_splits, static_cast<float*>(scratch), kNoAllocScratchBytes,
                                  status, stream);
}

}  // extern "C"
