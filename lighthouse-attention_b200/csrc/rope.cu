// Rotary position embedding for q and k in one pass (model harness; the
// reference applies RoPE in torchtitan's attention before the Lighthouse call,
// PATCH:700-737).  Adjacent pairs (x[2i], x[2i+1]) of each head row are
// rotated by the angle of table entry (position s, pair i):
//     (a, b) -> (a cos - b sin, a sin + b cos)          (inverse: sin -> -sin)
// computed in fp32 and rounded once to the storage type, which is what the
// complex64 multiply of the PyTorch formulation does.  One thread per 16-byte
// chunk of a (b, s, h) row; the table is (S, D/2) pairs of fp32 (cos, sin).
#include "lh_common.cuh"

namespace lh {

template <class T>
__global__ void __launch_bounds__(256)
rope_kernel(const T* __restrict__ xq, const T* __restrict__ xk, T* __restrict__ oq, T* __restrict__ ok,
            const float2* __restrict__ table, FastDiv fd_h, FastDiv fd_s, int D, int cpr_shift, float sin_sign,
            uint32_t n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const T* x = blockIdx.y == 0 ? xq : xk;
  T* o = blockIdx.y == 0 ? oq : ok;
  for (uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks; gid += gridDim.x * blockDim.x) {
    const uint32_t row = gid >> cpr_shift;          // (b * S + s) * H + h
    const int c = (int)(gid & ((1u << cpr_shift) - 1)) * VEC;
    uint32_t bs, h, b, s;
    fd_h.divmod(row, bs, h);
    fd_s.divmod(bs, b, s);
    float v[VEC], r[VEC];
    load16(x + (size_t)row * D + c, v);
    const float2* tb = table + (size_t)s * (D / 2) + c / 2;
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      const float2 cs = __ldg(tb + e / 2);
      const float sn = cs.y * sin_sign;
      r[e] = v[e] * cs.x - v[e + 1] * sn;
      r[e + 1] = v[e] * sn + v[e + 1] * cs.x;
    }
    store16(o + (size_t)row * D + c, r);
  }
}

int rope_apply(const void* xq, const void* xk, void* oq, void* ok, const float* table, int dtype, int B, int S,
               int H, int D, int inverse, cudaStream_t st) {
  const int esz = dtype == LH_DTYPE_BF16 ? 2 : 4;
  const int cpr = D * esz / 16;
  if (D % 2 || (D * esz) % 16 || (cpr & (cpr - 1))) { set_error("rope: D*elem_size/16 must be a power of two"); return LH_ERR_ARG; }
  const long long total = (long long)B * S * H * cpr;
  if (total >= (1LL << 31)) { set_error("rope: tensor too large"); return LH_ERR_SHAPE; }
  int cs = 0;
  while ((1 << cs) < cpr) ++cs;
  const uint32_t n = (uint32_t)total;
  long long g = (total + 255) / 256;
  if (g > 148LL * 16) g = 148LL * 16;
  dim3 grid((unsigned)(g < 1 ? 1 : g), 2);
  FastDiv fh(H), fs(S);
  const float sign = inverse ? -1.f : 1.f;
  if (dtype == LH_DTYPE_BF16)
    rope_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)xq, (const __nv_bfloat16*)xk,
        (__nv_bfloat16*)oq, (__nv_bfloat16*)ok, (const float2*)table, fh, fs, D, cs, sign, n);
  else
    rope_kernel<float><<<grid, 256, 0, st>>>((const float*)xq, (const float*)xk, (float*)oq, (float*)ok,
        (const float2*)table, fh, fs, D, cs, sign, n);
  return check_launch("rope_kernel");
}

}  // namespace lh
