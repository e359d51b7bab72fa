// sparse_attention_kernel instances for __half KV.
#include "attn_dispatch.cuh"

namespace linattn {
cudaError_t launch_sparse_attention_f16(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream) {
  return launch_dg<__half>(p, D, G, grid, stream);
}
cudaError_t launch_sparse_attention_mma_f16(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                          int box_rows, int D, int* counter, int64_t n_items, cudaStream_t stream) {
  return launch_mma<__half>(p, tmk, tmv, box_rows, D, counter, n_items, stream);
}
int tile_rows_f16(int D) { return tile_rows<__half>(D); }
}  // namespace linattn
