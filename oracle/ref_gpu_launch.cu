// TEST INFRASTRUCTURE ONLY (oracle). CUDA launcher for the reference's own
// selection kernel source, compiled by nvcc with the reference's NVRTC flags
// (--use_fast_math, src/lighthouse_selection_cuda.py:339-343) so that GPU
// tests can compare the product kernel against the reference kernel itself,
// fast-math level offsets included.  The kernel source is rendered from the
// reference by build_ref.py into oracle/_ref/ and passed in as REF_SRC.
#include <cuda_runtime.h>

#include REF_SRC

extern "C" int ref_gpu_topk(const float* scores_qk, const float* scores_kq,
                            unsigned int* keys_out, int* values_out,
                            int B, int KVH, int S_tot, int S_sel,
                            int num_levels, int pooling_factor, int N,
                            int n_chunk_coarsest, int num_sel_idx_chunk,
                            int num_tiles, void* stream) {
  // shared memory size as in src/lighthouse_selection_cuda.py:404-408
  const int smem = 128 / 2 * 4 * 4 + 128 * 4 + 128 * 4 * 2;
  dim3 grid(B * KVH, num_tiles, 1);
  lighthouse_selection_chunked_topk_kernel<<<grid, 128, smem, (cudaStream_t)stream>>>(
      scores_qk, scores_kq, keys_out, values_out,
      KVH * S_tot, S_tot, 1, KVH * S_tot, S_tot, 1,
      KVH * S_sel, S_sel, 1,
      num_levels, pooling_factor, KVH, N,
      n_chunk_coarsest, num_sel_idx_chunk);
  return (int)cudaGetLastError();
}
