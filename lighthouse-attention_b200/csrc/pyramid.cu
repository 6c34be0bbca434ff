// Pyramid + norm-score kernel (one streaming pass over q, k, v).
//
// Computes what DialatedLighthouseNormScorer.forward does with ~10 ATen
// passes (reference src/lighthouse_selection.py:589-616):
//   score_l0[t,h]  = dtype(||x[t,h,:]||_2)              for x = q (qk) and k (kq)
//   pooled_l[j,h]  = dtype(mean_{i<p^l} x[j*p^l + i, h])  for q, k, v, l = 1..L-1
//   score_l[j,h]   = max_{i<p^l} score_l0[j*p^l + i, h]
// Level 0 is never copied: consumers address raw tokens directly.
//
// Work decomposition: a CTA owns TPC consecutive tokens (a multiple of
// p^(L-1)) of one batch row and all H heads.  Each thread owns one
// (head, 16-byte column chunk) and walks the tokens in order, so every level's
// mean is a sequential fp32 sum over raw tokens and every load is a coalesced
// 128-bit load (a warp reads 512 contiguous bytes per token).  Scores are
// staged in shared memory and written as contiguous per-head runs.
#include "lh_common.cuh"


namespace lh {

constexpr int kPyrThreads = 128;

constexpr int kPyrU = 4;                 // tokens per load batch
constexpr int kPyrStages = 4;            // batches in flight per thread

__device__ __forceinline__ void pyr_cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void pyr_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// blockIdx.z selects the tensor (0 = q, 1 = k, 2 = v): each thread carries the
// level accumulators of one tensor only, and q / k threads also produce that
// tensor's norm scores.  Loads go through a per-thread ring in shared memory:
// kPyrStages batches of kPyrU tokens (16 tokens, 256 bytes per thread) are in
// flight by cp.async while the oldest batch is reduced.  A thread only reads
// back the chunks it copied itself, so the ring needs no barrier, and the
// in-flight data holds no registers (more CTAs per SM than a register
// double buffer: 6 per SM at 80 registers for L <= 3).
template <class T, int D, int LV>
__global__ void __launch_bounds__(kPyrThreads, LV <= 3 ? 6 : 4)
pyramid_score_kernel(const T* __restrict__ xq, const T* __restrict__ xk, const T* __restrict__ xv,
                     int S, int H, int p_shift, int tpc,
                     T* __restrict__ pq, T* __restrict__ pk, T* __restrict__ pv,
                     float* __restrict__ sqk, float* __restrict__ skq, Pyramid pyr, int S_pool) {
  constexpr int VEC = Vec16<T>::N;       // elements per 16-byte chunk
  constexpr int LPH = D / VEC;           // lanes per head row
  constexpr int U = kPyrU;
  constexpr int NST = kPyrStages;
  static_assert(LPH <= 32 && (32 % LPH) == 0, "head row must fit a warp segment");
  extern __shared__ __align__(16) uint8_t s_dyn[];
  const uint4* ring = reinterpret_cast<const uint4*>(s_dyn);                    // [NST][U][threads]
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(s_dyn);
  float* s_scores = reinterpret_cast<float*>(s_dyn + (size_t)NST * U * kPyrThreads * 16);  // [H][tpc_tot]
  const int which = blockIdx.z;
  const T* x = which == 0 ? xq : (which == 1 ? xk : xv);
  T* px = which == 0 ? pq : (which == 1 ? pk : pv);
  float* sc = which == 0 ? sqk : skq;
  const bool scored = which < 2;
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * tpc;
  const int ntok = min(tpc, S - t0);
  int tpc_tot = 0;
  int lvl_base[LV];
#pragma unroll
  for (int l = 0; l < LV; ++l) { lvl_base[l] = tpc_tot; tpc_tot += tpc >> (l * p_shift); }

  const int pairs = H * LPH;
  const int pairs_padded = (pairs + 31) & ~31;
  for (int pr = threadIdx.x; pr < pairs_padded; pr += blockDim.x) {
    const bool active = pr < pairs;
    const int h = active ? pr / LPH : 0;
    const int c = (pr % LPH) * VEC;
    const T* src = x + (((size_t)b * S + t0) * H + h) * D + c;
    const size_t tok_stride = (size_t)H * D;
    float acc[LV][VEC];
    float mx[LV];
#pragma unroll
    for (int l = 1; l < LV; ++l) {
      mx[l] = -INFINITY;
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[l][e] = 0.f;
    }
    // batch n of this thread's tokens -> ring stage n % NST (zero-filled past the end)
    auto issue = [&](int n) {
      const int st = n % NST;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = n * U + u;
        const bool ok = active && i < ntok;
        pyr_cp16(ring_s + (uint32_t)(((st * U + u) * kPyrThreads + threadIdx.x) * 16),
                 ok ? (const void*)(src + (size_t)i * tok_stride) : (const void*)x, ok);
      }
    };
    auto process = [&](int n) {
      const int st = n % NST, i0 = n * U;
      float buf[U][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) unpack16(ring[(st * U + u) * kPyrThreads + threadIdx.x], buf[u], (const T*)nullptr);
      // the U tokens' norm reductions run side by side (independent shuffle chains)
      float nrms[U];
      if (scored) {
        float ss[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          ss[u] = 0.f;
#pragma unroll
          for (int e = 0; e < VEC; ++e) ss[u] = fmaf(buf[u][e], buf[u][e], ss[u]);
        }
#pragma unroll
        for (int m = LPH / 2; m > 0; m >>= 1) {
#pragma unroll
          for (int u = 0; u < U; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], m, LPH);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) nrms[u] = round_to(sqrtf(ss[u]), (const T*)nullptr);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u;
        const float nrm = scored ? nrms[u] : 0.f;
        if (i >= ntok || !active) continue;
        if (scored && c == 0) s_scores[h * tpc_tot + i] = nrm;
#pragma unroll
        for (int l = 1; l < LV; ++l) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[l][e] += buf[u][e];
          mx[l] = fmaxf(mx[l], nrm);
          const int sh = l * p_shift;
          if (((i + 1) & ((1 << sh) - 1)) == 0) {
            const int j = i >> sh;                              // pooled index inside this CTA
            const float inv = 1.0f / (float)(1 << sh);          // exact: power of two
            float o[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) { o[e] = acc[l][e] * inv; acc[l][e] = 0.f; }
            const size_t prow = ((size_t)b * H + h) * S_pool + (pyr.off[l] - S) + (t0 >> sh) + j;
            store16(px + prow * D + c, o);
            if (scored && c == 0) s_scores[h * tpc_tot + lvl_base[l] + j] = mx[l];
            mx[l] = -INFINITY;
          }
        }
      }
    };
    // One commit group per batch (empty past the end), so that "batch n has
    // landed" is "at most NST-1 groups pending" at trip n.  A stage is refilled
    // only after this thread has reduced the values read from it.
    const int nb = (ntok + U - 1) / U;
#pragma unroll
    for (int n = 0; n < NST; ++n) {
      if (n < nb) issue(n);
      pyr_commit();
    }
    for (int n = 0; n < nb; ++n) {
      asm volatile("cp.async.wait_group %0;" ::"n"(NST - 1) : "memory");
      process(n);
      if (n + NST < nb) issue(n + NST);
      pyr_commit();
    }
  }
  if (!scored) return;
  __syncthreads();
  // Contiguous per-(head, level) runs of fp32 scores.
  for (int h = 0; h < H; ++h) {
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      const int n = ntok >> (l * p_shift);
      float* g = sc + ((size_t)b * H + h) * pyr.total + pyr.off[l] + (t0 >> (l * p_shift));
      for (int j = threadIdx.x; j < n; j += blockDim.x) g[j] = s_scores[h * tpc_tot + lvl_base[l] + j];
    }
  }
}

template <class T, int D, int LV>
static int launch_pyr(const void* xq, const void* xk, const void* xv, int B, int S, int H, int p,
                      void* pq, void* pk, void* pv, float* sqk, float* skq, cudaStream_t st) {
  int shift = 0;
  while ((1 << shift) < p) ++shift;
  const int G = 1 << (shift * (LV - 1));
  const int tpc = G >= 64 ? G : 64;
  Pyramid pyr; pyr.init(S, LV, p);
  const int S_pool = pyr.total - S;
  int tpc_tot = 0;
  for (int l = 0; l < LV; ++l) tpc_tot += tpc >> (l * shift);
  const size_t ring = (size_t)kPyrStages * kPyrU * kPyrThreads * 16;
  const size_t smem = ring + (size_t)H * tpc_tot * sizeof(float);
  if (smem > 200 * 1024) { set_error("pyramid: H*tpc too large for shared memory"); return LH_ERR_SHAPE; }
  auto kern = pyramid_score_kernel<T, D, LV>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((S + tpc - 1) / tpc, B, 3);
  kern<<<grid, kPyrThreads, smem, st>>>((const T*)xq, (const T*)xk, (const T*)xv, S, H, shift, tpc,
                                        (T*)pq, (T*)pk, (T*)pv, sqk, skq, pyr, S_pool);
  return check_launch("pyramid_score_kernel");
}

template <class T, int D>
static int dispatch_L(const void* xq, const void* xk, const void* xv, int B, int S, int H, int L, int p,
                      void* pq, void* pk, void* pv, float* sqk, float* skq, cudaStream_t st) {
  switch (L) {
    case 2: return launch_pyr<T, D, 2>(xq, xk, xv, B, S, H, p, pq, pk, pv, sqk, skq, st);
    case 3: return launch_pyr<T, D, 3>(xq, xk, xv, B, S, H, p, pq, pk, pv, sqk, skq, st);
    case 4: return launch_pyr<T, D, 4>(xq, xk, xv, B, S, H, p, pq, pk, pv, sqk, skq, st);
    case 5: return launch_pyr<T, D, 5>(xq, xk, xv, B, S, H, p, pq, pk, pv, sqk, skq, st);
    case 6: return launch_pyr<T, D, 6>(xq, xk, xv, B, S, H, p, pq, pk, pv, sqk, skq, st);
  }
  set_error("pyramid: L must be in [2, 6], got %d", L);
  return LH_ERR_SHAPE;
}

int pyramid_score_fwd(const void* xq, const void* xk, const void* xv, int dtype, int B, int S, int H,
                      int D, int L, int p, void* pq, void* pk, void* pv, float* sqk, float* skq,
                      cudaStream_t st) {
  if (dtype == LH_DTYPE_BF16) {
    if (D == 128) return dispatch_L<__nv_bfloat16, 128>(xq, xk, xv, B, S, H, L, p, pq, pk, pv, sqk, skq, st);
    if (D == 64) return dispatch_L<__nv_bfloat16, 64>(xq, xk, xv, B, S, H, L, p, pq, pk, pv, sqk, skq, st);
  } else if (dtype == LH_DTYPE_F32) {
    if (D == 128) return dispatch_L<float, 128>(xq, xk, xv, B, S, H, L, p, pq, pk, pv, sqk, skq, st);
    if (D == 64) return dispatch_L<float, 64>(xq, xk, xv, B, S, H, L, p, pq, pk, pv, sqk, skq, st);
  }
  set_error("pyramid: unsupported dtype %d / head dim %d", dtype, D);
  return LH_ERR_ARG;
}

}  // namespace lh
