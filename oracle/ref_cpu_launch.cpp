// TEST INFRASTRUCTURE ONLY (oracle). Host-thread launcher for the reference's
// selection kernel source compiled as C++ (see ref_cpu_shim.h).  The kernel
// source itself is not in this repository: build_ref.py renders it from the
// reference at build time into oracle/_ref/ and passes its path as REF_SRC.
//
// Launch geometry follows the reference host wrapper
// (src/lighthouse_selection_cuda.py:404-423): grid (B*KVH, NUM_TILES),
// block 128, one block at a time here.
#include "ref_cpu_shim.h"
#include <thread>
#include <vector>

thread_local ref_dim3 threadIdx;
thread_local ref_dim3 blockIdx;
std::barrier<>* ref_block_barrier = nullptr;
uint32_t ref_xchg[1024];
alignas(16) char smem_raw[1 << 16];

#include REF_SRC

extern "C" int ref_cpu_topk(const float* scores_qk, const float* scores_kq,
                            unsigned int* keys_out, int* values_out,
                            int B, int KVH, int S_tot, int S_sel,
                            int num_levels, int pooling_factor, int N,
                            int n_chunk_coarsest, int num_sel_idx_chunk,
                            int num_tiles) {
  const int nthreads = 128;
  std::barrier<> bar(nthreads);
  ref_block_barrier = &bar;
  std::vector<std::thread> pool;
  for (int t = 0; t < nthreads; ++t) {
    pool.emplace_back([=, &bar]() {
      threadIdx = {(unsigned)t, 0, 0};
      for (int bx = 0; bx < B * KVH; ++bx) {
        for (int by = 0; by < num_tiles; ++by) {
          blockIdx = {(unsigned)bx, (unsigned)by, 0};
          lighthouse_selection_chunked_topk_kernel(
              scores_qk, scores_kq, keys_out, values_out,
              KVH * S_tot, S_tot, 1, KVH * S_tot, S_tot, 1,
              KVH * S_sel, S_sel, 1,
              num_levels, pooling_factor, KVH, N,
              n_chunk_coarsest, num_sel_idx_chunk);
          bar.arrive_and_wait();
        }
      }
    });
  }
  for (auto& th : pool) th.join();
  ref_block_barrier = nullptr;
  return 0;
}
