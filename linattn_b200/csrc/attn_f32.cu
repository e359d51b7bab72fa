// sparse_attention_kernel instances for float KV.
#include "attn_dispatch.cuh"

namespace linattn {
cudaError_t launch_sparse_attention_f32(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream) {
  return launch_dg<float>(p, D, G, grid, stream);
}
int tile_rows_f32(int D) { return tile_rows<float>(D); }
}  // namespace linattn
