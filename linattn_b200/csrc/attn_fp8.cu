// sparse_attention_kernel instances for fp8e4m3 KV.
#include "attn_dispatch.cuh"

namespace linattn {
cudaError_t launch_sparse_attention_fp8(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream) {
  return launch_dg<fp8e4m3>(p, D, G, grid, stream);
}
cudaError_t launch_sparse_attention_mma_fp8(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                            int box_rows, int D, int* counter, int64_t n_items, cudaStream_t stream) {
  return launch_mma<fp8e4m3>(p, tmk, tmv, box_rows, D, counter, n_items, stream);
}
int tile_rows_fp8(int D) { return tile_rows<fp8e4m3>(D); }
}  // namespace linattn
