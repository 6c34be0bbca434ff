// Hierarchical qk/kq chunked top-k selection, one warp per (b, h, tile).
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
//  * One warp holds the 128 (score, index) pairs in registers, element i at
//    lane i%32, register i/32.  Stages with j >= 32 are register
//    compare-exchanges inside a thread, stages with j < 32 are xor shuffles.
//    No shared memory, no __syncthreads inside the sort.
//  * The qk sort carries each candidate's kq score as payload, so the kq sort
//    of the qk rejects needs no dependent global load; the next batch's
//    scores are prefetched while the current batch sorts.
//  * The reference writes (ordered-float key, value) pairs and sorts them
//    globally.  In the defined domain every candidate of every level is
//    written exactly once and the keys order the output as a post-order walk
//    of the refinement tree (children by position, then the refined parent,
//    whose key c_l*(idx+1) - 2^(1-level) sorts after all its descendants).
//    So this kernel only records which entries were refined (one bitmap per
//    level in shared memory), sizes each coarsest entry's subtree, takes a
//    warp prefix sum and writes the final position-ordered indices directly,
//    plus the inverse map used by the scatter and un-pool kernels.  The
//    per-row torch.sort / torch.gather of the reference disappear.
#include "lh_common.cuh"

namespace lh {

constexpr int kSelTopk = 128;
constexpr int kSelHalf = 64;
constexpr float kNegBig = -1e6f;   // placeholder score (reference :191-194, :227)

// Comparator stages of the descending bitonic network, branch-free.
// NP = number of payload arrays moved with the key (1: index; 2: index + score).
// Stages with j < 32 exchange across lanes (xor shuffles); k and j may be
// run-time values there.
template <int NP>
__device__ __forceinline__ void shuffle_stage(int k, int j, int lane, float (&key)[4], float (&pf)[4],
                                              int (&ix)[4]) {
  // Integer predicates on purpose: the same logic written with bool ternaries
  // compiles to a form about four times slower per stage on this target.
  const int lower = (lane & j) == 0;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = lane + 32 * r;
    const int desc = (i & k) == 0;
    const float o = __shfl_xor_sync(0xffffffffu, key[r], j);
    const int oi = __shfl_xor_sync(0xffffffffu, ix[r], j);
    float op = 0.f;
    if (NP > 1) op = __shfl_xor_sync(0xffffffffu, pf[r], j);
    // lower partner keeps the larger value when descending; strict compares keep ties in place
    const int lt = key[r] < o, gt = key[r] > o;
    const int swap = (lower ^ desc) ? gt : lt;
    key[r] = swap ? o : key[r];
    ix[r] = swap ? oi : ix[r];
    if (NP > 1) pf[r] = swap ? op : pf[r];
  }
}

// Stages with j >= 32 exchange registers inside a thread; K and J are
// compile-time so that the register indices are constants.
template <int NP, int K, int J>
__device__ __forceinline__ void register_stage(int lane, float (&key)[4], float (&pf)[4], int (&ix)[4]) {
  constexpr int rr = J >> 5;
#pragma unroll
  for (int lo = 0; lo < 4; ++lo) {
    if (lo & rr) continue;
    const int hi = lo | rr;
    const int i_lo = lane + 32 * lo;
    const int desc = (i_lo & K) == 0;
    const float a = key[lo], b = key[hi];
    const int lt = a < b, gt = a > b;
    const int swap = desc ? lt : gt;
    key[lo] = swap ? b : a;
    key[hi] = swap ? a : b;
    const int ia = ix[lo], ib = ix[hi];
    ix[lo] = swap ? ib : ia;
    ix[hi] = swap ? ia : ib;
    if (NP > 1) {
      const float pa = pf[lo], pb = pf[hi];
      pf[lo] = swap ? pb : pa;
      pf[hi] = swap ? pa : pb;
    }
  }
}

struct SortSet2 { float key[4]; float pf[4]; int ix[4]; };   // qk sort: key qk, payload kq score + index
struct SortSet1 { float key[4]; float pf[4]; int ix[4]; };   // kq sort: key kq, payload index

// The network as compact loops: stages with j < 32 take k and j at run time
// (only the register index is unrolled); the three stages with j >= 32 are
// spelled out.  A fully unrolled network is tens of KB of straight-line code
// executed by one warp per SM, which stalls on instruction fetch.
// NETS = 1: the kq set only; 2: the qk set only; 3: both, stage by stage
// (two independent networks for instruction-level parallelism).
template <int NETS>
__device__ __forceinline__ void shuffle_stage2(int k, int j, int lane, SortSet2& a, SortSet1& b) {
  if (NETS & 2) shuffle_stage<2>(k, j, lane, a.key, a.pf, a.ix);
  if (NETS & 1) shuffle_stage<1>(k, j, lane, b.key, b.pf, b.ix);
}
template <int NETS, int K, int J>
__device__ __forceinline__ void register_stage2(int lane, SortSet2& a, SortSet1& b) {
  if (NETS & 2) register_stage<2, K, J>(lane, a.key, a.pf, a.ix);
  if (NETS & 1) register_stage<1, K, J>(lane, b.key, b.pf, b.ix);
}

template <int NETS>
__device__ __forceinline__ void bitonic128_sets(int lane, SortSet2& a, SortSet1& b) {
#pragma unroll 1
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll 1
    for (int j = k >> 1; j > 0; j >>= 1) shuffle_stage2<NETS>(k, j, lane, a, b);
  }
  register_stage2<NETS, 64, 32>(lane, a, b);
#pragma unroll 1
  for (int j = 16; j > 0; j >>= 1) shuffle_stage2<NETS>(64, j, lane, a, b);
  register_stage2<NETS, 128, 64>(lane, a, b);
  register_stage2<NETS, 128, 32>(lane, a, b);
#pragma unroll 1
  for (int j = 16; j > 0; j >>= 1) shuffle_stage2<NETS>(128, j, lane, a, b);
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

__global__ void __launch_bounds__(32)
select_topk_kernel(const float* __restrict__ sq_all, const float* __restrict__ sk_all, SelGeom g,
                   Pyramid pyr, int32_t* __restrict__ indices, int32_t* __restrict__ inverse) {
  extern __shared__ uint32_t s_dyn[];
  int* s_parent = reinterpret_cast<int*>(s_dyn);            // [128]
  int* s_bmoff = reinterpret_cast<int*>(s_dyn + kSelTopk);  // [8] bitmap word offset per level
  int* s_lvloff = s_bmoff + 8;                              // [8] pyramid offset per level
  uint32_t* s_bm = s_dyn + kSelTopk + 16;                   // refinement bitmaps
  const int lane = threadIdx.x;
  const int bh = blockIdx.x / g.T;
  const int tile = blockIdx.x % g.T;
  const float* sq = sq_all + (size_t)bh * g.S_tot;
  const float* sk = sk_all + (size_t)bh * g.S_tot;
  for (int w = lane; w < g.bm_words; w += 32) s_bm[w] = 0u;
  for (int i = lane; i < kSelTopk; i += 32) s_parent[i] = -1;
  if (lane < 8) { s_bmoff[lane] = g.bm_word_off[lane]; s_lvloff[lane] = pyr.off[lane]; }
  __syncwarp();

  const int pmask = g.p - 1;
  for (int lev = g.L; lev >= 2; --lev) {
    const int lvl_off = s_lvloff[lev - 1];
    const int K_end = (g.N >> ((lev - 1) * g.shift)) - 1;    // last entry of this level
    const int ncand = (lev == g.L) ? g.ncc : g.p * kSelTopk;
    const int tile_start = tile * g.ncc;
    auto cand = [&](int c) -> int {
      if (c >= ncand) return -1;
      if (lev == g.L) return tile_start + c;
      const int pv = s_parent[c >> g.shift];
      if (pv < 0) return -1;
      const int kidx = pv * g.p + (c & pmask);
      return (kidx > K_end) ? -1 : kidx;
    };
    auto valid = [&](int kidx) { return kidx >= 0 && kidx <= K_end; };

    // qk set: regs 0,1 = running top-64 by qk, regs 2,3 = the batch being sorted.
    // kq set: regs 0,1 = running top-64 by kq, regs 2,3 = the qk rejects.
    SortSet2 qk;
    SortSet1 kq;
#pragma unroll
    for (int r = 0; r < 4; ++r) { qk.key[r] = kNegBig; qk.pf[r] = kNegBig; qk.ix[r] = -1; kq.key[r] = kNegBig; kq.pf[r] = 0.f; kq.ix[r] = -1; }

    const int nb = (ncand + kSelHalf - 1) / kSelHalf;
    int nidx[2];
    float nq[2], nk[2];
    auto fetch = [&](int bt) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        nidx[r] = cand(bt * kSelHalf + lane + 32 * r);
        nq[r] = valid(nidx[r]) ? __ldg(sq + lvl_off + nidx[r]) : kNegBig;
        nk[r] = valid(nidx[r]) ? __ldg(sk + lvl_off + nidx[r]) : kNegBig;
      }
    };
    auto take = [&]() {
#pragma unroll
      for (int r = 0; r < 2; ++r) { qk.ix[2 + r] = nidx[r]; qk.key[2 + r] = nq[r]; qk.pf[2 + r] = nk[r]; }
    };
    fetch(0);
    take();
    if (nb > 1) fetch(1);
    // qk sort of batch 0 (reference :203-232)
    bitonic128_sets<2>(lane, qk, kq);
    for (int bt = 0; bt < nb; ++bt) {
      // kq set for batch bt: its top-64 and the qk rejects (reference :242-250)
#pragma unroll
      for (int r = 0; r < 2; ++r) { kq.key[2 + r] = qk.pf[2 + r]; kq.ix[2 + r] = qk.ix[2 + r]; }
      if (bt + 1 < nb) {
        take();                                  // batch bt+1 joins the qk top-64
        if (bt + 2 < nb) fetch(bt + 2);
        // kq sort of batch bt and qk sort of batch bt+1 are independent: run them together
        bitonic128_sets<3>(lane, qk, kq);
      } else {
        bitonic128_sets<1>(lane, qk, kq);
      }
    }
    int tki[2], ix[2];
    tki[0] = kq.ix[0]; tki[1] = kq.ix[1];
    ix[0] = qk.ix[0]; ix[1] = qk.ix[1];
    __syncwarp();
    // Parents of the next level: [top-64 by qk ; top-64 by kq] (reference :324-327)
    s_parent[lane] = ix[0];
    s_parent[32 + lane] = ix[1];
    s_parent[64 + lane] = tki[0];
    s_parent[96 + lane] = tki[1];
    const int start = tile * (g.ncc << ((g.L - lev) * g.shift));
    const int kept[4] = {ix[0], ix[1], tki[0], tki[1]};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int rel = kept[r] - start;
      if (kept[r] >= 0) atomicOr(&s_bm[s_bmoff[lev] + (rel >> 5)], 1u << (rel & 31));
    }
    __syncwarp();
  }

  // ---- placement: post-order walk of each coarsest entry's refinement tree.
  // Stackless: children of (lev, idx) are (lev-1, idx*p .. idx*p+p-1), so the
  // walk descends to the first child of refined nodes, steps to the next
  // sibling, and climbs to (and emits) the parent after its last child.
  const int per_lane = g.ncc / 32;
  const int e0 = tile * g.ncc + lane * per_lane;
  auto walk = [&](int e, auto&& visit) {
    int lev = g.L, idx = e;
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
  for (int e = e0; e < e0 + per_lane; ++e) walk(e, [&](int, int) { ++count; });
  int incl = count;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, m);
    if (lane >= m) incl += v;
  }
  int slot = tile * g.chunk_len + incl - count;
  int32_t* out = indices + (size_t)bh * g.S_sel;
  int32_t* inv = inverse ? inverse + (size_t)bh * g.S_tot : nullptr;
  for (int e = e0; e < e0 + per_lane; ++e) {
    walk(e, [&](int lev, int idx) {
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
  const size_t smem = (kSelTopk + 16 + (size_t)g.bm_words) * sizeof(uint32_t);
  if (smem > 200 * 1024) { set_error("select: refinement bitmaps exceed shared memory"); return LH_ERR_SHAPE; }
  if (smem > 48 * 1024) cudaFuncSetAttribute(select_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (inverse) {
    cudaError_t e = cudaMemsetAsync(inverse, 0xff, sizeof(int32_t) * (size_t)B * H * g.S_tot, st);
    if (e != cudaSuccess) { set_error("select: memset inverse: %s", cudaGetErrorString(e)); return LH_ERR_LAUNCH; }
  }
  select_topk_kernel<<<B * H * g.T, 32, smem, st>>>(sqk, skq, g, pyr, indices, inverse);
  return check_launch("select_topk_kernel");
}

}  // namespace lh
