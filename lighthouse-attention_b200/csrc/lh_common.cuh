// Shared helpers for the Lighthouse B200 kernels (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/lighthouse_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "lighthouse_b200 is written for sm_100a (B200) only"
#endif

namespace lh {

// Thread-local error text; set by entry points before returning non-zero.
void set_error(const char* fmt, ...);

// Launch check used by every entry point after its kernel launches.
int check_launch(const char* what);

__host__ __device__ inline long long ipow(long long b, int e) {
  long long r = 1;
  while (e-- > 0) r *= b;
  return r;
}

// Pyramid geometry of one (b,h) row.  Level l (0 = raw tokens) holds N/p^l
// entries and starts at offset(l) = sum_{j<l} N/p^j of the concatenated
// pyramid (reference: src/lighthouse_selection.py:600-614).
struct Pyramid {
  int N, L, p;
  int off[8];   // start of level l
  int len[8];   // entries in level l
  int total;    // S_tot
  __host__ __device__ void init(int N_, int L_, int p_) {
    N = N_; L = L_; p = p_;
    int acc = 0;
    for (int l = 0; l < 8; ++l) {
      int n = (l < L) ? (int)(N / ipow(p, l)) : 0;
      off[l] = acc; len[l] = n; acc += n;
    }
    total = acc;
  }
};

// S_sel: the selected-sequence length (reference:
// src/lighthouse_selection_cuda.py:346-357).
__host__ __device__ inline long long sel_len(long long N, int L, int p, int k) {
  long long t = 0;
  for (int level = L; level >= 1; --level)
    t += (level == L) ? N / ipow(p, level - 1) : (long long)p * k;
  return t;
}

// Division of non-negative 31-bit integers by a launch-invariant divisor with
// one multiply-high, an add and a shift (Granlund & Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994): with s = ceil(log2 d)
// and m = floor(2^32 (2^s - d) / d) + 1, n / d = (umulhi(n, m) + n) >> s for
// 0 <= n < 2^31.  Built on the host, used in row-mover index arithmetic.
struct FastDiv {
  uint32_t d, m, s;
  __host__ __device__ FastDiv() : d(1), m(0), s(0) {}
  __host__ explicit FastDiv(uint32_t div) : d(div) {
    s = 0;
    while ((1ull << s) < div) ++s;
    m = (uint32_t)((((1ull << s) - div) << 32) / div + 1);
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#ifdef __CUDA_ARCH__
    const uint32_t hi = __umulhi(n, m);
#else
    const uint32_t hi = (uint32_t)(((uint64_t)n * m) >> 32);
#endif
    return (hi + n) >> s;
  }
  __host__ __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
    q = div(n);
    r = n - q * d;
  }
};

template <class T> struct Vec16;
template <> struct Vec16<__nv_bfloat16> { static constexpr int N = 8; };
template <> struct Vec16<float> { static constexpr int N = 4; };

__device__ __forceinline__ void load16(const __nv_bfloat16* p, float* f) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x; f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void load16(const float* p, float* f) {
  float4 u = __ldg(reinterpret_cast<const float4*>(p));
  f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
}
// 16 raw bytes as VEC floats (the pointer argument only selects the element type).
__device__ __forceinline__ void unpack16(const uint4& u, float* f, const __nv_bfloat16*) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x; f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void unpack16(const uint4& u, float* f, const float*) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void store16(__nv_bfloat16* p, const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store16(float* p, const float* f) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}

// Round a float to the storage type and back (the reference returns scores in
// the input dtype before converting them to fp32).
__device__ __forceinline__ float round_to(float x, const __nv_bfloat16*) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float round_to(float x, const float*) { return x; }

}  // namespace lh
