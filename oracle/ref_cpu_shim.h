// TEST INFRASTRUCTURE ONLY (oracle). Lets the reference's own selection
// kernel source (the CUDA C string built by `_make_kernel_source` in
// src/lighthouse_selection_cuda.py:7-331 of the reference) compile as plain
// C++ and run on host threads: one std::thread per CUDA thread of a block,
// __syncthreads as a block-wide barrier, __shfl_xor_sync as an exchange
// through a shared slot array between two barriers.  Blocks run one after
// another, so the kernel's `extern __shared__` array can be a single global.
//
// Nothing here is product code; the product path never links it.
#pragma once
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <algorithm>

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __shared__
#define __restrict__ __restrict

struct ref_dim3 { unsigned x, y, z; };
extern thread_local ref_dim3 threadIdx;
extern thread_local ref_dim3 blockIdx;
extern std::barrier<> *ref_block_barrier;
extern uint32_t ref_xchg[1024];

inline void __syncthreads() { ref_block_barrier->arrive_and_wait(); }

inline unsigned int __float_as_uint(float f) { unsigned int u; std::memcpy(&u, &f, 4); return u; }
inline float __int2float_rn(int i) { return (float)i; }
template <class T> inline T __ldg(const T* p) { return *p; }
using std::min;

template <class T>
inline T __shfl_xor_sync(unsigned, T v, int lane_mask) {
  static_assert(sizeof(T) == 4, "32-bit shuffles only");
  const unsigned t = threadIdx.x;
  uint32_t bits; std::memcpy(&bits, &v, 4);
  ref_xchg[t] = bits;
  __syncthreads();
  // __shfl_xor_sync exchanges inside a 32-lane warp
  uint32_t other = ref_xchg[(t & ~31u) | ((t & 31u) ^ (unsigned)lane_mask)];
  __syncthreads();
  T r; std::memcpy(&r, &other, 4);
  return r;
}
