// sparse_attention_kernel instances for __nv_bfloat16 KV.
#include "attn_dispatch.cuh"

namespace linattn {
cudaError_t launch_sparse_attention_bf16(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream) {
  return launch_dg<__nv_bfloat16>(p, D, G, grid, stream);
}
cudaError_t launch_sparse_attention_mma_bf16(const AttnParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                          int box_rows, int D, int* counter, int64_t n_items, cudaStream_t stream) {
  return launch_mma<__nv_bfloat16>(p, tmk, tmv, box_rows, D, counter, n_items, stream);
}
int tile_rows_bf16(int D) { return tile_rows<__nv_bfloat16>(D); }
}  // namespace linattn
