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

template <class T, int D, int LV>
__global__ void __launch_bounds__(kPyrThreads)
pyramid_score_kernel(const T* __restrict__ xq, const T* __restrict__ xk, const T* __restrict__ xv,
                     int S, int H, int p_shift, int tpc,
                     T* __restrict__ pq, T* __restrict__ pk, T* __restrict__ pv,
                     float* __restrict__ sqk, float* __restrict__ skq, Pyramid pyr, int S_pool) {
  constexpr int VEC = Vec16<T>::N;       // elements per 16-byte chunk
  constexpr int LPH = D / VEC;           // lanes per head row
  static_assert(LPH <= 32 && (32 % LPH) == 0, "head row must fit a warp segment");
  extern __shared__ float s_scores[];    // [2][H][tpc_tot]
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * tpc;
  const int ntok = min(tpc, S - t0);
  int tpc_tot = 0;
  int lvl_base[LV];
#pragma unroll
  for (int l = 0; l < LV; ++l) { lvl_base[l] = tpc_tot; tpc_tot += tpc >> (l * p_shift); }
  float* sb_q = s_scores;
  float* sb_k = s_scores + H * tpc_tot;

  const int pairs = H * LPH;
  const int pairs_padded = (pairs + 31) & ~31;
  for (int pr = threadIdx.x; pr < pairs_padded; pr += blockDim.x) {
    const bool active = pr < pairs;
    const int h = active ? pr / LPH : 0;
    const int c = (pr % LPH) * VEC;
    const size_t row0 = ((size_t)b * S + t0) * H + h;     // (b, t0, h) row
    float acc_q[LV][VEC], acc_k[LV][VEC], acc_v[LV][VEC];
    float mx_q[LV], mx_k[LV];
#pragma unroll
    for (int l = 1; l < LV; ++l) {
      mx_q[l] = -INFINITY; mx_k[l] = -INFINITY;
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc_q[l][e] = acc_k[l][e] = acc_v[l][e] = 0.f;
    }
    constexpr int U = 4;  // tokens in flight per thread
    for (int i0 = 0; i0 < ntok; i0 += U) {
      float fq[U][VEC], fk[U][VEC], fv[U][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (active && i0 + u < ntok) {
          const size_t off = (row0 + (size_t)(i0 + u) * H) * D + c;
          load16(xq + off, fq[u]); load16(xk + off, fk[u]); load16(xv + off, fv[u]);
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) fq[u][e] = fk[u][e] = fv[u][e] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u;
        float ssq = 0.f, ssk = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) { ssq = fmaf(fq[u][e], fq[u][e], ssq); ssk = fmaf(fk[u][e], fk[u][e], ssk); }
#pragma unroll
        for (int m = LPH / 2; m > 0; m >>= 1) {
          ssq += __shfl_xor_sync(0xffffffffu, ssq, m, LPH);
          ssk += __shfl_xor_sync(0xffffffffu, ssk, m, LPH);
        }
        if (i >= ntok || !active) continue;
        const float nq = round_to(sqrtf(ssq), (const T*)nullptr);
        const float nk = round_to(sqrtf(ssk), (const T*)nullptr);
        if (c == 0) { sb_q[h * tpc_tot + i] = nq; sb_k[h * tpc_tot + i] = nk; }
#pragma unroll
        for (int l = 1; l < LV; ++l) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) { acc_q[l][e] += fq[u][e]; acc_k[l][e] += fk[u][e]; acc_v[l][e] += fv[u][e]; }
          mx_q[l] = fmaxf(mx_q[l], nq); mx_k[l] = fmaxf(mx_k[l], nk);
          const int sh = l * p_shift;
          if (((i + 1) & ((1 << sh) - 1)) == 0) {
            const int j = i >> sh;                              // pooled index inside this CTA
            const float inv = 1.0f / (float)(1 << sh);          // exact: power of two
            float oq[VEC], ok[VEC], ov[VEC];
#pragma unroll
            for (int e = 0; e < VEC; ++e) { oq[e] = acc_q[l][e] * inv; ok[e] = acc_k[l][e] * inv; ov[e] = acc_v[l][e] * inv;
                                            acc_q[l][e] = acc_k[l][e] = acc_v[l][e] = 0.f; }
            const size_t prow = ((size_t)b * H + h) * S_pool + (pyr.off[l] - S) + (t0 >> sh) + j;
            store16(pq + prow * D + c, oq); store16(pk + prow * D + c, ok); store16(pv + prow * D + c, ov);
            if (c == 0) { sb_q[h * tpc_tot + lvl_base[l] + j] = mx_q[l]; sb_k[h * tpc_tot + lvl_base[l] + j] = mx_k[l]; }
            mx_q[l] = -INFINITY; mx_k[l] = -INFINITY;
          }
        }
      }
    }
  }
  __syncthreads();
  // Contiguous per-(head, level) runs of fp32 scores.
  for (int h = 0; h < H; ++h) {
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      const int n = ntok >> (l * p_shift);
      float* gq = sqk + ((size_t)b * H + h) * pyr.total + pyr.off[l] + (t0 >> (l * p_shift));
      float* gk = skq + ((size_t)b * H + h) * pyr.total + pyr.off[l] + (t0 >> (l * p_shift));
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        gq[j] = sb_q[h * tpc_tot + lvl_base[l] + j];
        gk[j] = sb_k[h * tpc_tot + lvl_base[l] + j];
      }
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
  const size_t smem = (size_t)2 * H * tpc_tot * sizeof(float);
  if (smem > 200 * 1024) { set_error("pyramid: H*tpc too large for shared memory"); return LH_ERR_SHAPE; }
  auto kern = pyramid_score_kernel<T, D, LV>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((S + tpc - 1) / tpc, B);
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
