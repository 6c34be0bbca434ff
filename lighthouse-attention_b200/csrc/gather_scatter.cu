// Row movers around the attention: gather of selected pyramid rows, the
// deterministic fan-out scatter (forward + adjoint), the inverse map, and the
// un-pool backward.  All are HBM-bound row copies with 16-byte accesses; each
// thread owns one 16-byte chunk of a D-wide row.
#include "lh_common.cuh"

namespace lh {

constexpr int kRowThreads = 256;

// ---------------------------------------------------------------- gather
// out[bh, s] = idx < S ? raw[b, idx, h] : pooled[bh, idx - S]
// (reference src/lighthouse_selection.py:800-813)
template <class T>
__global__ void __launch_bounds__(kRowThreads)
gather_kernel(const T* __restrict__ raw0, const T* __restrict__ raw1, const T* __restrict__ raw2,
              const T* __restrict__ pool0, const T* __restrict__ pool1, const T* __restrict__ pool2,
              T* __restrict__ out0, T* __restrict__ out1, T* __restrict__ out2,
              const int32_t* __restrict__ indices, int H, int S, int D, int S_pool, int S_sel,
              long long n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const int cpr = D / VEC;
  const T* raw = blockIdx.y == 0 ? raw0 : (blockIdx.y == 1 ? raw1 : raw2);
  const T* pool = blockIdx.y == 0 ? pool0 : (blockIdx.y == 1 ? pool1 : pool2);
  T* out = blockIdx.y == 0 ? out0 : (blockIdx.y == 1 ? out1 : out2);
  if (out == nullptr) return;
  for (long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks;
       gid += (long long)gridDim.x * blockDim.x) {
    const long long row = gid / cpr;         // bh * S_sel + s
    const int c = (int)(gid % cpr) * VEC;
    const int bh = (int)(row / S_sel);
    const int idx = __ldg(indices + row);
    const T* src;
    if (idx < S) {
      const int b = bh / H, h = bh % H;
      src = raw + (((size_t)b * S + idx) * H + h) * D;
    } else {
      src = pool + ((size_t)bh * S_pool + (idx - S)) * D;
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * D + c) = __ldg(reinterpret_cast<const uint4*>(src + c));
  }
}

// ---------------------------------------------------------------- scatter (pull)
// out[bh, t] = sum_l attn[bh, inv(l, (t+1)/p^l - 1)] over levels whose item
// window [j*f + f - 1, j*f + 2f - 1) contains t (reference :408-459).
template <class T>
__global__ void __launch_bounds__(kRowThreads)
scatter_fwd_kernel(const T* __restrict__ attn, const int32_t* __restrict__ inverse, Pyramid pyr,
                   int D, int S_sel, int N_total, T* __restrict__ out, long long n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const int cpr = D / VEC;
  for (long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks;
       gid += (long long)gridDim.x * blockDim.x) {
    const long long row = gid / cpr;        // bh * N_total + t
    const int c = (int)(gid % cpr) * VEC;
    const int bh = (int)(row / N_total);
    const int t = (int)(row % N_total);
    const int32_t* inv = inverse + (size_t)bh * pyr.total;
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    int f = 1;
    for (int l = 0; l < pyr.L; ++l, f *= pyr.p) {
      const int j = (t + 1) / f - 1;
      if (j >= 0 && j < pyr.len[l]) {
        const int slot = __ldg(inv + pyr.off[l] + j);
        if (slot >= 0) {
          float v[VEC];
          load16(attn + ((size_t)bh * S_sel + slot) * D + c, v);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] += v[e];
        }
      }
    }
    store16(out + (size_t)row * D + c, acc);
  }
}

// ---------------------------------------------------------------- scatter adjoint
// dattn[bh, s] = sum over the item's window of dout[bh, pos] (reference :462-514)
template <class T>
__global__ void __launch_bounds__(kRowThreads)
scatter_bwd_kernel(const T* __restrict__ dout, const int32_t* __restrict__ indices, Pyramid pyr,
                   int D, int S_sel, int N_total, T* __restrict__ dattn, long long n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const int cpr = D / VEC;
  for (long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks;
       gid += (long long)gridDim.x * blockDim.x) {
    const long long row = gid / cpr;        // bh * S_sel + s
    const int c = (int)(gid % cpr) * VEC;
    const int bh = (int)(row / S_sel);
    const int idx = __ldg(indices + row);
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    if (idx >= 0) {
      int l = 0, f = 1;
      while (l + 1 < pyr.L && idx >= pyr.off[l + 1]) { ++l; f *= pyr.p; }
      if (idx < pyr.off[l] + pyr.len[l]) {
        const int first = (idx - pyr.off[l]) * f + f - 1;
        const T* src = dout + (size_t)bh * N_total * D + c;
        for (int i = 0; i < f; ++i) {
          const int pos = first + i;
          if (pos >= N_total) break;
          float v[VEC];
          load16(src + (size_t)pos * D, v);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] += v[e];
        }
      }
    }
    store16(dattn + (size_t)row * D + c, acc);
  }
}

// ---------------------------------------------------------------- inverse map
__global__ void inverse_kernel(const int32_t* __restrict__ indices, int S_sel, int S_tot,
                               int32_t* __restrict__ inverse, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int bh = (int)(i / S_sel);
    const int s = (int)(i % S_sel);
    const int idx = indices[i];
    if (idx >= 0 && idx < S_tot) inverse[(size_t)bh * S_tot + idx] = s;
  }
}

// ---------------------------------------------------------------- un-pool backward
// dx[b, t, h] = sum_l dsel[bh, inv(off_l + t/p^l)] / p^l   (autograd of :800-813, :604-606)
template <class T>
__global__ void __launch_bounds__(kRowThreads)
unpool_bwd_kernel(const T* __restrict__ d0, const T* __restrict__ d1, const T* __restrict__ d2,
                  T* __restrict__ o0, T* __restrict__ o1, T* __restrict__ o2,
                  const int32_t* __restrict__ inverse, Pyramid pyr, int H, int D, int S_sel,
                  long long n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const int cpr = D / VEC;
  const T* dsel = blockIdx.y == 0 ? d0 : (blockIdx.y == 1 ? d1 : d2);
  T* dx = blockIdx.y == 0 ? o0 : (blockIdx.y == 1 ? o1 : o2);
  if (dx == nullptr) return;
  const int S = pyr.N;
  for (long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks;
       gid += (long long)gridDim.x * blockDim.x) {
    const long long row = gid / cpr;        // (b * S + t) * H + h
    const int c = (int)(gid % cpr) * VEC;
    const int h = (int)(row % H);
    const long long bt = row / H;
    const int t = (int)(bt % S);
    const int b = (int)(bt / S);
    const int bh = b * H + h;
    const int32_t* inv = inverse + (size_t)bh * pyr.total;
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    int f = 1;
    for (int l = 0; l < pyr.L; ++l, f *= pyr.p) {
      const int j = t / f;
      if (j < pyr.len[l]) {
        const int slot = __ldg(inv + pyr.off[l] + j);
        if (slot >= 0) {
          float v[VEC];
          load16(dsel + ((size_t)bh * S_sel + slot) * D + c, v);
          const float sc = 1.0f / (float)f;
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[e] = fmaf(v[e], sc, acc[e]);
        }
      }
    }
    store16(dx + (size_t)row * D + c, acc);
  }
}

static int grid_for(long long n) {
  long long g = (n + kRowThreads - 1) / kRowThreads;
  const long long cap = 148LL * 16;
  return (int)(g < cap ? (g < 1 ? 1 : g) : cap);
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int gather_selected(const void* qr, const void* kr, const void* vr, const void* qp, const void* kp,
                    const void* vp, int dtype, int B, int S, int H, int D, int S_pool,
                    const int32_t* indices, int S_sel, void* qs, void* ks, void* vs, cudaStream_t st) {
  const int esz = dtype == LH_DTYPE_BF16 ? 2 : 4;
  if ((D * esz) % 16) { set_error("gather: D*elem must be a multiple of 16 bytes"); return LH_ERR_ARG; }
  const void* ptrs[] = {qr, kr, vr, qp, kp, vp, qs, ks, vs};
  for (const void* p : ptrs) if (p && !aligned16(p)) { set_error("gather: pointers must be 16-byte aligned"); return LH_ERR_ARG; }
  const long long n = (long long)B * H * S_sel * (D * esz / 16);
  dim3 grid(grid_for(n), 3);
  if (dtype == LH_DTYPE_BF16) {
    using T = __nv_bfloat16;
    gather_kernel<T><<<grid, kRowThreads, 0, st>>>((const T*)qr, (const T*)kr, (const T*)vr, (const T*)qp,
        (const T*)kp, (const T*)vp, (T*)qs, (T*)ks, (T*)vs, indices, H, S, D, S_pool, S_sel, n);
  } else {
    using T = float;
    gather_kernel<T><<<grid, kRowThreads, 0, st>>>((const T*)qr, (const T*)kr, (const T*)vr, (const T*)qp,
        (const T*)kp, (const T*)vp, (T*)qs, (T*)ks, (T*)vs, indices, H, S, D, S_pool, S_sel, n);
  }
  return check_launch("gather_kernel");
}

int scatter_fwd(const void* attn, const int32_t* inverse, int dtype, int B, int H, int S_sel, int D,
                int N_shard, int N_total, int L, int p, void* out, cudaStream_t st) {
  Pyramid pyr; pyr.init(N_shard, L, p);
  const int esz = dtype == LH_DTYPE_BF16 ? 2 : 4;
  if (!aligned16(attn) || !aligned16(out) || (D * esz) % 16) { set_error("scatter_fwd: alignment"); return LH_ERR_ARG; }
  const long long n = (long long)B * H * N_total * (D * esz / 16);
  if (dtype == LH_DTYPE_BF16)
    scatter_fwd_kernel<__nv_bfloat16><<<grid_for(n), kRowThreads, 0, st>>>((const __nv_bfloat16*)attn, inverse, pyr, D, S_sel, N_total, (__nv_bfloat16*)out, n);
  else
    scatter_fwd_kernel<float><<<grid_for(n), kRowThreads, 0, st>>>((const float*)attn, inverse, pyr, D, S_sel, N_total, (float*)out, n);
  return check_launch("scatter_fwd_kernel");
}

int scatter_bwd(const void* dout, const int32_t* indices, int dtype, int B, int H, int S_sel, int D,
                int N_shard, int N_total, int L, int p, void* dattn, cudaStream_t st) {
  Pyramid pyr; pyr.init(N_shard, L, p);
  const int esz = dtype == LH_DTYPE_BF16 ? 2 : 4;
  if (!aligned16(dout) || !aligned16(dattn) || (D * esz) % 16) { set_error("scatter_bwd: alignment"); return LH_ERR_ARG; }
  const long long n = (long long)B * H * S_sel * (D * esz / 16);
  if (dtype == LH_DTYPE_BF16)
    scatter_bwd_kernel<__nv_bfloat16><<<grid_for(n), kRowThreads, 0, st>>>((const __nv_bfloat16*)dout, indices, pyr, D, S_sel, N_total, (__nv_bfloat16*)dattn, n);
  else
    scatter_bwd_kernel<float><<<grid_for(n), kRowThreads, 0, st>>>((const float*)dout, indices, pyr, D, S_sel, N_total, (float*)dattn, n);
  return check_launch("scatter_bwd_kernel");
}

int build_inverse(const int32_t* indices, int B, int H, int S_sel, int S_tot, int32_t* inverse, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(inverse, 0xff, sizeof(int32_t) * (size_t)B * H * S_tot, st);
  if (e != cudaSuccess) { set_error("build_inverse: %s", cudaGetErrorString(e)); return LH_ERR_LAUNCH; }
  const long long n = (long long)B * H * S_sel;
  inverse_kernel<<<grid_for(n), kRowThreads, 0, st>>>(indices, S_sel, S_tot, inverse, n);
  return check_launch("inverse_kernel");
}

int unpool_bwd(const void* dq, const void* dk, const void* dv, const int32_t* inverse, int dtype, int B,
               int S, int H, int D, int L, int p, int S_sel, void* dxq, void* dxk, void* dxv, cudaStream_t st) {
  Pyramid pyr; pyr.init(S, L, p);
  const int esz = dtype == LH_DTYPE_BF16 ? 2 : 4;
  if ((D * esz) % 16) { set_error("unpool_bwd: D*elem must be a multiple of 16 bytes"); return LH_ERR_ARG; }
  const long long n = (long long)B * S * H * (D * esz / 16);
  dim3 grid(grid_for(n), 3);
  if (dtype == LH_DTYPE_BF16) {
    using T = __nv_bfloat16;
    unpool_bwd_kernel<T><<<grid, kRowThreads, 0, st>>>((const T*)dq, (const T*)dk, (const T*)dv, (T*)dxq, (T*)dxk, (T*)dxv, inverse, pyr, H, D, S_sel, n);
  } else {
    using T = float;
    unpool_bwd_kernel<T><<<grid, kRowThreads, 0, st>>>((const T*)dq, (const T*)dk, (const T*)dv, (T*)dxq, (T*)dxk, (T*)dxv, inverse, pyr, H, D, S_sel, n);
  }
  return check_launch("unpool_bwd_kernel");
}

}  // namespace lh
