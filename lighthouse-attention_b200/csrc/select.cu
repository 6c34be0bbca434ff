// Hierarchical qk/kq chunked top-k selection, one 256-thread CTA per (b, h, tile).
//
// Semantics are those of the reference kernel
// lighthouse_selection_chunked_topk_kernel (src/lighthouse_selection_cuda.py:114-330)
// followed by its stable sort + gather (:425-427).  The result must be
// bit-identical, ties included, so the comparator network is the same
// 128-wide bitonic network (:41-110: stages k = 2..128, j = k/2..1, direction
// desc = (i & k) == 0, swaps only on strict inequality) applied in the same
// batch order and slot layout (:198-258).  The comparator network is an
// algorithm that has to be alike; its execution here is different:
//
//  * Two 128-thread networks run side by side: warps 0-3 hold the qk set
//    (element i in thread i: score, index and the candidate's kq score as
//    payload), warps 4-7 the kq set.  The kq sort of batch b's qk rejects and
//    the qk sort of batch b+1 are independent and run at the same time on
//    different warps; the rejects cross over through shared memory, so the
//    kq sort needs no dependent global load.  Stages with j < 32 are xor
//    shuffles, the three with j >= 32 go through shared memory under a
//    128-thread named barrier.  The next batch's scores are prefetched while
//    the current one sorts.
//  * The reference writes (ordered-float key, value) pairs and sorts them
//    globally.  In the defined domain every candidate of every level is
//    written exactly once and the keys order the output as a post-order walk
//    of the refinement tree (children by position, then the refined parent,
//    whose key c_l*(idx+1) - 2^(1-level) sorts after all its descendants).
//    So this kernel only records which entries were refined (one bitmap per
//    level in shared memory), sizes each coarsest entry's subtree, takes a
//    block prefix sum and writes the final position-ordered indices directly,
//    plus the inverse map used by the scatter and un-pool kernels.  The
//    per-row torch.sort / torch.gather of the reference disappear.
#include "lh_common.cuh"

namespace lh {

constexpr int kSelTopk = 128;
constexpr int kSelHalf = 64;
constexpr int kSelThreads = 256;
constexpr float kNegBig = -1e6f;   // placeholder score (reference :191-194, :227)

// One element of a 128-wide set: sort key, payload score (qk set: the
// candidate's kq score) and index.
struct SelElem { float key; float pf; int ix; };

// Shared-memory exchange buffers of one set: one per stage with j >= 32
// (k = 64 / j = 32, k = 128 / j = 64, k = 128 / j = 32).  Each buffer is
// written once per network and read after the group barrier; by the next
// network's write to it every thread has passed two later barriers.
struct SelXchg { float key[3][kSelTopk]; float pf[3][kSelTopk]; int ix[3][kSelTopk]; };

// Compare-exchange of element t with element t ^ j (value o) in the stage
// of bitonic block size k: the lower partner keeps the larger value when
// descending; strict compares leave ties in place.  Integer predicates, as
// bool ternaries compile to a slower form on this target.
template <bool PF>
__device__ __forceinline__ void cmp_swap(int t, int k, int j, SelElem& e, float ok, float op, int oi) {
  const int lower = (t & j) == 0, desc = (t & k) == 0;
  const int lt = e.key < ok, gt = e.key > ok;
  const int swap = (lower ^ desc) ? gt : lt;
  e.key = swap ? ok : e.key;
  e.ix = swap ? oi : e.ix;
  if (PF) e.pf = swap ? op : e.pf;
}

template <bool PF>
__device__ __forceinline__ void shfl_stage(int t, int k, int j, SelElem& e) {
  const float ok = __shfl_xor_sync(0xffffffffu, e.key, j);
  const int oi = __shfl_xor_sync(0xffffffffu, e.ix, j);
  const float op = PF ? __shfl_xor_sync(0xffffffffu, e.pf, j) : 0.f;
  cmp_swap<PF>(t, k, j, e, ok, op, oi);
}

template <bool PF>
__device__ __forceinline__ void smem_stage(int t, int k, int j, int buf, int bar_id, SelElem& e, SelXchg* x) {
  x->key[buf][t] = e.key;
  x->ix[buf][t] = e.ix;
  if (PF) x->pf[buf][t] = e.pf;
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(kSelTopk) : "memory");
  const int o = t ^ j;
  cmp_swap<PF>(t, k, j, e, x->key[buf][o], PF ? x->pf[buf][o] : 0.f, x->ix[buf][o]);
}

// The whole 128-wide descending network on the calling 128-thread group,
// fully unrolled (one element per thread keeps it a few hundred instructions).
template <bool PF>
__device__ __forceinline__ void bitonic128(int t, int bar_id, SelElem& e, SelXchg* x) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) shfl_stage<PF>(t, k, j, e);
  }
  smem_stage<PF>(t, 64, 32, 0, bar_id, e, x);
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) shfl_stage<PF>(t, 64, j, e);
  smem_stage<PF>(t, 128, 64, 1, bar_id, e, x);
  smem_stage<PF>(t, 128, 32, 2, bar_id, e, x);
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) shfl_stage<PF>(t, 128, j, e);
}

struct SelGeom {
  int N, L, p, shift, T, ncc, S_tot, S_sel, chunk_len;
  int bm_word_off[8];   // bitmap word offset for reference level `lev` (2..L)
  int bm_words;
};

// Reference level `lev` (1 = raw tokens, L = coarsest) is pyramid level lev-1.
__device__ __forceinline__ bool refined(const uint32_t* bm, const int* bm_off, const SelGeom& g, int lev, int idx,
                                        int tile) {
  if (lev < 2) return false;
  const int start = tile * (g.ncc << ((g.L - lev) * g.shift));
  const int rel = idx - start;
  return (bm[bm_off[lev] + (rel >> 5)] >> (rel & 31)) & 1u;
}

__global__ void __launch_bounds__(kSelThreads)
select_topk_kernel(const float* __restrict__ sq_all, const float* __restrict__ sk_all, SelGeom g,
                   Pyramid pyr, int32_t* __restrict__ indices, int32_t* __restrict__ inverse) {
  extern __shared__ __align__(16) uint32_t s_dyn[];
  SelXchg* s_x = reinterpret_cast<SelXchg*>(s_dyn);                   // [2]: qk group, kq group
  float* s_rej_pf = reinterpret_cast<float*>(s_x + 2);                 // [2][64] qk rejects: kq score
  int* s_rej_ix = reinterpret_cast<int*>(s_rej_pf + 2 * kSelHalf);     // [2][64] qk rejects: index
  int* s_parent = s_rej_ix + 2 * kSelHalf;                             // [128]
  int* s_bmoff = s_parent + kSelTopk;                                  // [8] bitmap word offset per level
  int* s_lvloff = s_bmoff + 8;                                         // [8] pyramid offset per level
  int* s_scan = s_lvloff + 8;                                          // [8] per-warp totals
  uint32_t* s_bm = reinterpret_cast<uint32_t*>(s_scan + 8);            // refinement bitmaps
  const int tid = threadIdx.x;
  const int grp = tid >> 7;                       // 0: qk set, 1: kq set
  const int t = tid & 127;                        // element of the set
  const int bar_id = 1 + grp;
  const int bh = blockIdx.x / g.T;
  const int tile = blockIdx.x % g.T;
  const float* sq = sq_all + (size_t)bh * g.S_tot;
  const float* sk = sk_all + (size_t)bh * g.S_tot;
  for (int w = tid; w < g.bm_words; w += kSelThreads) s_bm[w] = 0u;
  if (tid < kSelTopk) s_parent[tid] = -1;
  if (tid < 8) { s_bmoff[tid] = g.bm_word_off[tid]; s_lvloff[tid] = pyr.off[tid]; }
  __syncthreads();

  const int pmask = g.p - 1;
  for (int lev = g.L; lev >= 2; --lev) {
    const int lvl_off = s_lvloff[lev - 1];
    const int K_end = (g.N >> ((lev - 1) * g.shift)) - 1;    // last entry of this level
    const int ncand = (lev == g.L) ? g.ncc : g.p * kSelTopk;
    const int tile_start = tile * g.ncc;
    // qk elements 0..63: running top-64 by qk, 64..127: the batch being sorted.
    // kq elements 0..63: running top-64 by kq, 64..127: the qk rejects.
    SelElem e;
    e.key = kNegBig;
    e.pf = grp == 0 ? kNegBig : 0.f;
    e.ix = -1;
    const int nb = (ncand + kSelHalf - 1) / kSelHalf;
    // qk threads 64..127 fetch candidate bt * 64 + (t - 64) of each batch
    int nidx = -1;
    float nq = kNegBig, nk = kNegBig;
    auto fetch = [&](int bt) {
      const int c = bt * kSelHalf + t - kSelHalf;
      int kidx = -1;
      if (c < ncand) {
        if (lev == g.L) {
          kidx = tile_start + c;
        } else {
          const int pv = s_parent[c >> g.shift];
          if (pv >= 0) kidx = pv * g.p + (c & pmask);
        }
      }
      nidx = -1; nq = kNegBig; nk = kNegBig;
      if (kidx >= 0 && kidx <= K_end) {
        nidx = kidx;
        nq = __ldg(sq + lvl_off + kidx);
        nk = __ldg(sk + lvl_off + kidx);
      }
    };
    const bool loader = grp == 0 && t >= kSelHalf;
    if (loader) {
      fetch(0);
      e.ix = nidx; e.key = nq; e.pf = nk;        // batch 0 joins the qk set
      if (nb > 1) fetch(1);
    }
    if (grp == 0) bitonic128<true>(t, bar_id, e, &s_x[0]);     // qk sort of batch 0 (reference :203-232)
    for (int bt = 0; bt < nb; ++bt) {
      // the qk rejects of batch bt (elements 64..127) cross to the kq set (reference :242-250)
      if (loader) { s_rej_pf[(bt & 1) * kSelHalf + t - kSelHalf] = e.pf; s_rej_ix[(bt & 1) * kSelHalf + t - kSelHalf] = e.ix; }
      __syncthreads();
      if (grp == 1 && t >= kSelHalf) {
        e.key = s_rej_pf[(bt & 1) * kSelHalf + t - kSelHalf];
        e.ix = s_rej_ix[(bt & 1) * kSelHalf + t - kSelHalf];
      }
      if (grp == 0) {
        if (bt + 1 < nb) {
          if (loader) {
            e.ix = nidx; e.key = nq; e.pf = nk;  // batch bt+1 joins the qk top-64
            if (bt + 2 < nb) fetch(bt + 2);
          }
          bitonic128<true>(t, bar_id, e, &s_x[0]);
        }
      } else {
        bitonic128<false>(t, bar_id, e, &s_x[1]);
      }
    }
    __syncthreads();                              // every read of s_parent for this level is done
    // Parents of the next level: [top-64 by qk ; top-64 by kq] (reference :324-327)
    if (t < kSelHalf) {
      s_parent[grp * kSelHalf + t] = e.ix;
      const int start = tile * (g.ncc << ((g.L - lev) * g.shift));
      const int rel = e.ix - start;
      if (e.ix >= 0) atomicOr(&s_bm[s_bmoff[lev] + (rel >> 5)], 1u << (rel & 31));
    }
    __syncthreads();
  }

  // ---- placement: post-order walk of each coarsest entry's refinement tree.
  // Stackless: children of (lev, idx) are (lev-1, idx*p .. idx*p+p-1), so the
  // walk descends to the first child of refined nodes, steps to the next
  // sibling, and climbs to (and emits) the parent after its last child.
  const int per = (g.ncc + kSelThreads - 1) / kSelThreads;
  const int e0 = tile * g.ncc + min(tid * per, g.ncc);
  const int e1 = tile * g.ncc + min(tid * per + per, g.ncc);
  auto walk = [&](int en, auto&& visit) {
    int lev = g.L, idx = en;
    while (lev >= 2 && refined(s_bm, s_bmoff, g, lev, idx, tile)) { idx <<= g.shift; --lev; }
    while (true) {
      visit(lev, idx);
      if (lev == g.L) break;
      if ((idx & pmask) != pmask) {
        ++idx;
        while (lev >= 2 && refined(s_bm, s_bmoff, g, lev, idx, tile)) { idx <<= g.shift; --lev; }
      } else {
        idx >>= g.shift;
        ++lev;
      }
    }
  };
  int count = 0;
  for (int en = e0; en < e1; ++en) walk(en, [&](int, int) { ++count; });
  // block exclusive prefix sum of the counts (thread order = entry order)
  const int lane = tid & 31, warp = tid >> 5;
  int incl = count;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, m);
    if (lane >= m) incl += v;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += s_scan[w];
  int slot = tile * g.chunk_len + before + incl - count;
  int32_t* out = indices + (size_t)bh * g.S_sel;
  int32_t* inv = inverse ? inverse + (size_t)bh * g.S_tot : nullptr;
  for (int en = e0; en < e1; ++en) {
    walk(en, [&](int lev, int idx) {
      const int pidx = idx + s_lvloff[lev - 1];
      out[slot] = pidx;
      if (inv) inv[pidx] = slot;
      ++slot;
    });
  }
}

// Host-side domain check; mirrors the reference asserts (CU:370-375, 385, 391)
// and adds the conditions under which the reference kernel is well defined.
int select_geometry(int S, int L, int p, int k, SelGeom* g, Pyramid* pyr) {
  if (L < 2 || L > 7) { set_error("select: num_levels must be in [2, 7], got %d", L); return LH_ERR_SHAPE; }
  if (p < 2 || (p & (p - 1))) { set_error("select: pooling_factor must be a power of 2 >= 2, got %d", p); return LH_ERR_SHAPE; }
  if (k % 128) { set_error("select: topk must be a multiple of 128, got %d", k); return LH_ERR_SHAPE; }
  if (k / 2 < p) { set_error("select: topk/2 must be >= pooling_factor"); return LH_ERR_SHAPE; }
  const long long G = ipow(p, L - 1);
  if (S % G) { set_error("select: S=%d must be a multiple of p^(L-1)=%lld", S, G); return LH_ERR_SHAPE; }
  const int T = k / 128;
  const long long C = S / G;
  if (C % T) { set_error("select: coarsest length %lld not divisible by k/128=%d (reference kernel undefined)", C, T); return LH_ERR_SHAPE; }
  const int ncc = (int)(C / T);
  if (ncc < 128) { set_error("select: N_CHUNK_COARSEST=%d must be >= 128 (reference asserts, CU:391)", ncc); return LH_ERR_SHAPE; }
  if (ncc % 64) { set_error("select: N_CHUNK_COARSEST=%d must be a multiple of 64 (reference kernel undefined)", ncc); return LH_ERR_SHAPE; }
  pyr->init(S, L, p);
  g->N = S; g->L = L; g->p = p; g->T = T; g->ncc = ncc;
  g->shift = 0; while ((1 << g->shift) < p) ++g->shift;
  g->S_tot = pyr->total;
  g->S_sel = (int)sel_len(S, L, p, k);
  g->chunk_len = (int)sel_len(S / T, L, p, 128);
  int words = 0;
  for (int lev = 0; lev < 8; ++lev) g->bm_word_off[lev] = 0;
  for (int lev = 2; lev <= L; ++lev) {
    g->bm_word_off[lev] = words;
    words += (int)(((long long)ncc * ipow(p, L - lev) + 31) / 32);
  }
  g->bm_words = words;
  return LH_OK;
}

int select_topk(const float* sqk, const float* skq, int B, int H, int S, int L, int p, int k,
                int32_t* indices, int32_t* inverse, cudaStream_t st) {
  SelGeom g; Pyramid pyr;
  int rc = select_geometry(S, L, p, k, &g, &pyr);
  if (rc) return rc;
  const size_t smem = 2 * sizeof(SelXchg) + (4 * kSelHalf + kSelTopk + 24 + (size_t)g.bm_words) * sizeof(uint32_t);
  if (smem > 200 * 1024) { set_error("select: refinement bitmaps exceed shared memory"); return LH_ERR_SHAPE; }
  if (smem > 48 * 1024) cudaFuncSetAttribute(select_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (inverse) {
    cudaError_t e = cudaMemsetAsync(inverse, 0xff, sizeof(int32_t) * (size_t)B * H * g.S_tot, st);
    if (e != cudaSuccess) { set_error("select: memset inverse: %s", cudaGetErrorString(e)); return LH_ERR_LAUNCH; }
  }
  select_topk_kernel<<<B * H * g.T, kSelThreads, smem, st>>>(sqk, skq, g, pyr, indices, inverse);
  return check_launch("select_topk_kernel");
}

}  // namespace lh
