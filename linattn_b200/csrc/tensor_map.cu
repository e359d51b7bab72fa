// Cached TMA tensor-map encoding (cuTensorMapEncodeTiled through the runtime's
// driver entry point; the library links no libcuda symbol directly).
#include <cudaTypedefs.h>

#include <mutex>

#include "launchers.cuh"

namespace linattn {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct Entry {
  const void* base;
  int cu_dtype;
  int64_t inner, rows, stride_bytes;
  int box_inner, box_rows;
  bool used;
  CUtensorMap map;
};
std::mutex g_mu;
Entry g_cache[64];
int g_next = 0;

}  // namespace

// A map only encodes these values (no device state), so a cached one is valid
// whenever they match.
bool tensor_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType cu_dtype, int64_t inner, int64_t rows,
                   int64_t stride_bytes, int box_inner, int box_rows) {
  std::lock_guard<std::mutex> lock(g_mu);
  for (const Entry& e : g_cache)
    if (e.used && e.base == base && e.cu_dtype == static_cast<int>(cu_dtype) && e.inner == inner && e.rows == rows &&
        e.stride_bytes == stride_bytes && e.box_inner == box_inner && e.box_rows == box_rows) {
      *out = e.map;
      return true;
    }
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem_strides[2] = {1u, 1u};
  Entry& e = g_cache[g_next];
  const CUresult r = fn(&e.map, cu_dtype, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    e.used = false;
    return false;
  }
  e.base = base;
  e.cu_dtype = static_cast<int>(cu_dtype);
  e.inner = inner;
  e.rows = rows;
  e.stride_bytes = stride_bytes;
  e.box_inner = box_inner;
  e.box_rows = box_rows;
  e.used = true;
  *out = e.map;
  g_next = (g_next + 1) % 64;
  return true;
}

}  // namespace linattn
