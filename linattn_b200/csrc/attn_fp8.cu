// sparse_attention_kernel instances for fp8e4m3 KV.
#include "attn_dispatch.cuh"

namespace linattn {
cudaError_t launch_sparse_attention_fp8(const AttnParams& p, int D, int G, unsigned grid, cudaStream_t stream) {
  return launch_dg<fp8e4m3>(p, D, G, grid, stream);
}
int tile_rows_fp8(int D) { return tile_rows<fp8e4m3>(D); }
}  // namespace linattn
