// Causal attention backward (placeholder until the tcgen05 kernel lands).
#include "lh_common.cuh"
namespace lh {
size_t attn_bwd_workspace_size(int B, int H, int S_q, int S_kv, int D) {
  return (size_t)B * H * ((S_q + 127) / 128 * 128) * (D + 1) * sizeof(float) + 256;
}
int attn_bwd(const void*, const void*, const void*, const void*, const float*, const void*, int, int, int, int,
             int, int, float, void*, void*, void*, void*, size_t, cudaStream_t) {
  set_error("attn_bwd: not built");
  return LH_ERR_LAUNCH;
}
}  // namespace lh
