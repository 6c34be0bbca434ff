// Row movers around the attention: gather of selected pyramid rows, the
// deterministic fan-out scatter (forward + adjoint), the inverse map, and the
// un-pool backward.  All are HBM-bound row copies with 16-byte accesses; each
// thread owns one 16-byte chunk of a D-wide row.
#include <type_traits>

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
              const int32_t* __restrict__ indices, FastDiv fd_ssel, FastDiv fd_h, int S, int D, int S_pool,
              int cpr_shift, uint32_t n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const T* raw = blockIdx.y == 0 ? raw0 : (blockIdx.y == 1 ? raw1 : raw2);
  const T* pool = blockIdx.y == 0 ? pool0 : (blockIdx.y == 1 ? pool1 : pool2);
  T* out = blockIdx.y == 0 ? out0 : (blockIdx.y == 1 ? out1 : out2);
  if (out == nullptr) return;
  const int H = (int)fd_h.d;
  for (uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks; gid += gridDim.x * blockDim.x) {
    const uint32_t row = gid >> cpr_shift;           // bh * S_sel + s
    const int c = (int)(gid & ((1u << cpr_shift) - 1)) * VEC;
    const uint32_t bh = fd_ssel.div(row);
    const int idx = __ldg(indices + row);
    const T* src;
    if (idx < S) {
      uint32_t b, h;
      fd_h.divmod(bh, b, h);
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
template <class T, int LV>
__global__ void __launch_bounds__(kRowThreads)
scatter_fwd_kernel(const T* __restrict__ attn, const int32_t* __restrict__ inverse, Pyramid pyr, int p_shift,
                   int D, int S_sel, FastDiv fd_n, T* __restrict__ out, int cpr_shift, uint32_t n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  for (uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks; gid += gridDim.x * blockDim.x) {
    const uint32_t row = gid >> cpr_shift;          // bh * N_total + t
    const int c = (int)(gid & ((1u << cpr_shift) - 1)) * VEC;
    uint32_t bh, t;
    fd_n.divmod(row, bh, t);
    const int32_t* inv = inverse + (size_t)bh * pyr.total;
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    // all index loads first, then all row loads: no dependent chains between levels
    int slot[LV];
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      const int jj = (int)((t + 1) >> (l * p_shift)) - 1;
      slot[l] = (jj >= 0 && jj < pyr.len[l]) ? __ldg(inv + pyr.off[l] + jj) : -1;
    }
    float v[LV][VEC];
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      if (slot[l] >= 0) load16(attn + ((size_t)bh * S_sel + slot[l]) * D + c, v[l]);
      else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[l][e] = 0.f;
      }
    }
#pragma unroll
    for (int l = 0; l < LV; ++l) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] += v[l][e];
    }
    store16(out + (size_t)row * D + c, acc);
  }
}

// ---------------------------------------------------------------- grouped row kernels
// Scatter forward and un-pool backward over groups of kGroup consecutive
// tokens: one warp per (32 >> CS neighbouring b*h rows, kGroup tokens), one
// token of all the warp's heads per step, lanes = head x 16-byte chunk.
// Per token the output is
//     out(t) = v_0(t) + base(t),   base(t) = sum_{l >= 1} v_l(t)
// where v_l(t) is the (scaled) level-l row of the item containing t.  The
// level-l item changes only every p^l tokens, so base is rebuilt only at those
// steps; the level-0 row exists for a small fraction of tokens (those selected
// at full resolution).  The group's inverse-map entries are fetched once per
// level with coalesced loads and handed out by shuffles.
//   SHIFTED (scatter, reference :428-458): item jj_l(t) = (t+1)/p^l - 1, rows summed
//   !SHIFTED (un-pool backward of the mean pooling): jj_l(t) = t/p^l, rows scaled by 1/p^l
constexpr int kGroup = 16;
template <class T> struct TypeTag { using type = T; };

template <class T, int LV, int CS, bool SHIFTED>
__global__ void __launch_bounds__(kRowThreads)
grouped_rows_kernel(const T* __restrict__ s0, const T* __restrict__ s1, const T* __restrict__ s2,
                    T* __restrict__ o0, T* __restrict__ o1, T* __restrict__ o2,
                    const int32_t* __restrict__ inverse, Pyramid pyr, int p_shift, int D, int S_sel,
                    int N_out, int n_groups, int BH, int H, long long row_stride, long long bh_stride_b,
                    long long bh_stride_h) {
  constexpr int VEC = Vec16<T>::N;
  constexpr int LPH = 1 << CS;                  // lanes per head (16-byte chunks per row)
  constexpr int HPW = 32 / LPH;                 // heads per warp
  static_assert(LPH >= kGroup, "one level-0 entry per lane of a head");
  const T* src0 = blockIdx.y == 0 ? s0 : (blockIdx.y == 1 ? s1 : s2);
  T* dst0 = blockIdx.y == 0 ? o0 : (blockIdx.y == 1 ? o1 : o2);
  if (dst0 == nullptr) return;
  const int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int n_hg = BH / HPW;
  const int grp = w / n_hg;                     // head groups fastest: neighbouring warps, neighbouring rows
  if (grp >= n_groups) return;
  const int hh = lane / LPH, jl = lane % LPH;
  const int bh = (w - grp * n_hg) * HPW + hh;
  const int b = bh / H, h = bh - b * H;
  const int tg = grp * kGroup;
  const int c = jl * VEC;
  const int32_t* inv = inverse + (size_t)bh * pyr.total;
  const T* src = src0 + (size_t)bh * S_sel * D + c;
  T* dst = dst0 + b * bh_stride_b + h * bh_stride_h + c;

  // level-l entries of this group: item first_l + jl for jl < count_l
  int ent[LV];
#pragma unroll
  for (int l = 0; l < LV; ++l) {
    const int sh = l * p_shift;
    const int first = SHIFTED ? ((tg + 1) >> sh) - 1 : (tg >> sh);
    const int last = SHIFTED ? ((tg + kGroup) >> sh) - 1 : ((tg + kGroup - 1) >> sh);
    const int jj = first + jl;
    ent[l] = (jj <= last && jj >= 0 && jj < pyr.len[l]) ? __ldg(inv + pyr.off[l] + jj) : -1;
  }
  float base[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) base[e] = 0.f;
#pragma unroll
  for (int s = 0; s < kGroup; ++s) {
    const int t = tg + s;
    if (t >= N_out) break;
    // rebuild base where any level >= 1 starts a new item (warp-uniform)
    bool rebuild = s == 0;
#pragma unroll
    for (int l = 1; l < LV; ++l) rebuild |= (((SHIFTED ? t + 1 : t) & ((1 << (l * p_shift)) - 1)) == 0);
    if (rebuild) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) base[e] = 0.f;
#pragma unroll
      for (int l = 1; l < LV; ++l) {
        const int sh = l * p_shift;
        const int first = SHIFTED ? ((tg + 1) >> sh) - 1 : (tg >> sh);
        const int idx = (SHIFTED ? ((t + 1) >> sh) - 1 : (t >> sh)) - first;
        const int slot = __shfl_sync(0xffffffffu, ent[l], hh * LPH + idx);
        if (slot >= 0) {
          float v[VEC];
          load16(src + (size_t)slot * D, v);
          const float sc = SHIFTED ? 1.0f : 1.0f / (float)(1 << sh);
#pragma unroll
          for (int e = 0; e < VEC; ++e) base[e] = fmaf(v[e], sc, base[e]);
        }
      }
    }
    const int slot0 = __shfl_sync(0xffffffffu, ent[0], hh * LPH + s);
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = base[e];
    if (slot0 >= 0) {
      float v[VEC];
      load16(src + (size_t)slot0 * D, v);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] += v[e];
    }
    store16(dst + (size_t)t * row_stride, acc);
  }
}

// ---------------------------------------------------------------- scatter adjoint
// dattn[bh, s] = sum over the item's window of dout[bh, pos] (reference :462-514)
template <class T>
__global__ void __launch_bounds__(kRowThreads)
scatter_bwd_kernel(const T* __restrict__ dout, const int32_t* __restrict__ indices, Pyramid pyr, int p_shift,
                   int D, FastDiv fd_ssel, int N_total, T* __restrict__ dattn, int cpr_shift, uint32_t n_chunks,
                   int H, long long row_stride, long long b_stride, long long h_stride) {
  constexpr int VEC = Vec16<T>::N;
  for (uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks; gid += gridDim.x * blockDim.x) {
    const uint32_t row = gid >> cpr_shift;          // bh * S_sel + s
    const int c = (int)(gid & ((1u << cpr_shift) - 1)) * VEC;
    const uint32_t bh = fd_ssel.div(row);
    const int idx = __ldg(indices + row);
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    if (idx >= 0) {
      int l = 0, lvl_off = 0, lvl_len = pyr.len[0];
#pragma unroll
      for (int m = 1; m < 8; ++m)
        if (m < pyr.L && idx >= pyr.off[m]) { l = m; lvl_off = pyr.off[m]; lvl_len = pyr.len[m]; }
      if (idx < lvl_off + lvl_len) {
        const int f = 1 << (l * p_shift);
        const int first = (idx - lvl_off) * f + f - 1;
        const int last = min(first + f, N_total);
        const int b = (int)bh / H, h = (int)bh - b * H;
        const T* src = dout + b * b_stride + h * h_stride + c;
        // four independent loads in flight per trip; the fp32 sum keeps position order
        int pos = first;
        for (; pos + 4 <= last; pos += 4) {
          float v[4][VEC];
#pragma unroll
          for (int u = 0; u < 4; ++u) load16(src + (size_t)(pos + u) * row_stride, v[u]);
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[e] += v[u][e];
        }
        for (; pos < last; ++pos) {
          float v[VEC];
          load16(src + (size_t)pos * row_stride, v);
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
template <class T, int LV>
__global__ void __launch_bounds__(kRowThreads)
unpool_bwd_kernel(const T* __restrict__ d0, const T* __restrict__ d1, const T* __restrict__ d2,
                  T* __restrict__ o0, T* __restrict__ o1, T* __restrict__ o2,
                  const int32_t* __restrict__ inverse, Pyramid pyr, int p_shift, FastDiv fd_h, FastDiv fd_s,
                  int D, int S_sel, int cpr_shift, uint32_t n_chunks) {
  constexpr int VEC = Vec16<T>::N;
  const T* dsel = blockIdx.y == 0 ? d0 : (blockIdx.y == 1 ? d1 : d2);
  T* dx = blockIdx.y == 0 ? o0 : (blockIdx.y == 1 ? o1 : o2);
  if (dx == nullptr) return;
  const int H = (int)fd_h.d;
  for (uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x; gid < n_chunks; gid += gridDim.x * blockDim.x) {
    const uint32_t row = gid >> cpr_shift;          // (b * S + t) * H + h
    const int c = (int)(gid & ((1u << cpr_shift) - 1)) * VEC;
    uint32_t bt, h, b, t;
    fd_h.divmod(row, bt, h);
    fd_s.divmod(bt, b, t);
    const uint32_t bh = b * H + h;
    const int32_t* inv = inverse + (size_t)bh * pyr.total;
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    int slot[LV];
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      const int jj = (int)(t >> (l * p_shift));
      slot[l] = jj < pyr.len[l] ? __ldg(inv + pyr.off[l] + jj) : -1;
    }
    float v[LV][VEC];
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      if (slot[l] >= 0) load16(dsel + ((size_t)bh * S_sel + slot[l]) * D + c, v[l]);
      else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[l][e] = 0.f;
      }
    }
#pragma unroll
    for (int l = 0; l < LV; ++l) {
      const float sc = 1.0f / (float)(1 << (l * p_shift));
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = fmaf(v[l][e], sc, acc[e]);
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

// Calls f(std::integral_constant<int, L>) for L in [1, 7]; false otherwise.
template <class F>
static bool dispatch_levels(int L, F&& f) {
  switch (L) {
    case 1: f(std::integral_constant<int, 1>{}); return true;
    case 2: f(std::integral_constant<int, 2>{}); return true;
    case 3: f(std::integral_constant<int, 3>{}); return true;
    case 4: f(std::integral_constant<int, 4>{}); return true;
    case 5: f(std::integral_constant<int, 5>{}); return true;
    case 6: f(std::integral_constant<int, 6>{}); return true;
    case 7: f(std::integral_constant<int, 7>{}); return true;
  }
  return false;
}

// Launches grouped_rows_kernel when the geometry fits (16 or 32 chunks per
// row, heads divisible into warps); returns false otherwise.
template <bool SHIFTED>
static bool launch_grouped_rows(int dtype, int L, int cs, const void* s0, const void* s1, const void* s2, void* o0,
                                void* o1, void* o2, int n_tensors, const int32_t* inverse, const Pyramid& pyr,
                                int p_shift, int D, int S_sel, int N_out, int B, int H, long long row_stride,
                                long long bh_stride_b, long long bh_stride_h, cudaStream_t st) {
  if (cs != 4 && cs != 5) return false;
  const int hpw = 32 >> cs;
  if ((B * H) % hpw || (SHIFTED ? false : H % hpw)) return false;
  if (L < 1 || L > 7) return false;
  const int n_groups = (N_out + kGroup - 1) / kGroup;
  const long long threads = (long long)(B * H / hpw) * n_groups * 32;
  dim3 grid((unsigned)((threads + kRowThreads - 1) / kRowThreads), n_tensors);
  auto go = [&](auto lv) {
    constexpr int LV = decltype(lv)::value;
    auto run = [&](auto cs_c, auto t_tag) {
      constexpr int CS = decltype(cs_c)::value;
      using T = typename decltype(t_tag)::type;
      grouped_rows_kernel<T, LV, CS, SHIFTED><<<grid, kRowThreads, 0, st>>>(
          (const T*)s0, (const T*)s1, (const T*)s2, (T*)o0, (T*)o1, (T*)o2, inverse, pyr, p_shift, D, S_sel, N_out,
          n_groups, B * H, H, row_stride, bh_stride_b, bh_stride_h);
    };
    auto by_cs = [&](auto t_tag) {
      if (cs == 4) run(std::integral_constant<int, 4>{}, t_tag);
      else run(std::integral_constant<int, 5>{}, t_tag);
    };
    if (dtype == LH_DTYPE_BF16) by_cs(TypeTag<__nv_bfloat16>{});
    else by_cs(TypeTag<float>{});
  };
  return dispatch_levels(L, go);
}

static int log2i(int x) { int s = 0; while ((1 << s) < x) ++s; return s; }

// chunks of 16 bytes per row as a shift; rejects totals beyond 31 bits
static int row_geometry(const char* what, int dtype, int D, long long rows, int* cpr_shift, uint32_t* n) {
  const int esz = dtype == LH_DTYPE_BF16 ? 2 : 4;
  const int cpr = D * esz / 16;
  if ((D * esz) % 16 || (cpr & (cpr - 1))) { set_error("%s: D*elem_size/16 must be a power of two", what); return LH_ERR_ARG; }
  const long long total = rows * cpr;
  if (total >= (1LL << 31)) { set_error("%s: tensor too large (%lld 16-byte chunks)", what, total); return LH_ERR_SHAPE; }
  *cpr_shift = log2i(cpr);
  *n = (uint32_t)total;
  return LH_OK;
}

int gather_selected(const void* qr, const void* kr, const void* vr, const void* qp, const void* kp,
                    const void* vp, int dtype, int B, int S, int H, int D, int S_pool,
                    const int32_t* indices, int S_sel, void* qs, void* ks, void* vs, cudaStream_t st) {
  const void* ptrs[] = {qr, kr, vr, qp, kp, vp, qs, ks, vs};
  for (const void* p : ptrs) if (p && !aligned16(p)) { set_error("gather: pointers must be 16-byte aligned"); return LH_ERR_ARG; }
  int cs; uint32_t n;
  int rc = row_geometry("gather", dtype, D, (long long)B * H * S_sel, &cs, &n);
  if (rc) return rc;
  dim3 grid(grid_for(n), 3);
  FastDiv fs(S_sel), fh(H);
  if (dtype == LH_DTYPE_BF16) {
    using T = __nv_bfloat16;
    gather_kernel<T><<<grid, kRowThreads, 0, st>>>((const T*)qr, (const T*)kr, (const T*)vr, (const T*)qp,
        (const T*)kp, (const T*)vp, (T*)qs, (T*)ks, (T*)vs, indices, fs, fh, S, D, S_pool, cs, n);
  } else {
    using T = float;
    gather_kernel<T><<<grid, kRowThreads, 0, st>>>((const T*)qr, (const T*)kr, (const T*)vr, (const T*)qp,
        (const T*)kp, (const T*)vp, (T*)qs, (T*)ks, (T*)vs, indices, fs, fh, S, D, S_pool, cs, n);
  }
  return check_launch("gather_kernel");
}

// token_major = 0: out is (B, H, N_total, D); 1: out is (B, N_total, H, D), the
// layout the output projection reads (the transpose after the layer,
// lighthouse-attention.patch:737, becomes a view).
int scatter_fwd_layout(const void* attn, const int32_t* inverse, int dtype, int B, int H, int S_sel, int D,
                       int N_shard, int N_total, int L, int p, int token_major, void* out, cudaStream_t st) {
  Pyramid pyr; pyr.init(N_shard, L, p);
  if (!aligned16(attn) || !aligned16(out)) { set_error("scatter_fwd: pointers must be 16-byte aligned"); return LH_ERR_ARG; }
  int cs; uint32_t n;
  int rc = row_geometry("scatter_fwd", dtype, D, (long long)B * H * N_total, &cs, &n);
  if (rc) return rc;
  const long long row_stride = token_major ? (long long)H * D : D;
  const long long b_stride = (long long)H * N_total * D;
  const long long h_stride = token_major ? D : (long long)N_total * D;
  if (launch_grouped_rows<true>(dtype, L, cs, attn, nullptr, nullptr, out, nullptr, nullptr, 1, inverse, pyr,
                                log2i(p), D, S_sel, N_total, B, H, row_stride, b_stride, h_stride, st))
    return check_launch("scatter_fwd (grouped)");
  if (token_major) {
    set_error("scatter_fwd: the token-major layout needs 256- or 512-byte rows and B*H divisible by the heads per warp");
    return LH_ERR_SHAPE;
  }
  FastDiv fn(N_total);
  auto go = [&](auto lv) {
    constexpr int LV = decltype(lv)::value;
    if (dtype == LH_DTYPE_BF16)
      scatter_fwd_kernel<__nv_bfloat16, LV><<<grid_for(n), kRowThreads, 0, st>>>((const __nv_bfloat16*)attn, inverse, pyr, log2i(p), D, S_sel, fn, (__nv_bfloat16*)out, cs, n);
    else
      scatter_fwd_kernel<float, LV><<<grid_for(n), kRowThreads, 0, st>>>((const float*)attn, inverse, pyr, log2i(p), D, S_sel, fn, (float*)out, cs, n);
  };
  if (!dispatch_levels(L, go)) { set_error("scatter_fwd: L must be in [1, 7]"); return LH_ERR_SHAPE; }
  return check_launch("scatter_fwd");
}

int scatter_fwd(const void* attn, const int32_t* inverse, int dtype, int B, int H, int S_sel, int D,
                int N_shard, int N_total, int L, int p, void* out, cudaStream_t st) {
  return scatter_fwd_layout(attn, inverse, dtype, B, H, S_sel, D, N_shard, N_total, L, p, 0, out, st);
}

// token_major as for scatter_fwd_layout, for dout.
int scatter_bwd_layout(const void* dout, const int32_t* indices, int dtype, int B, int H, int S_sel, int D,
                       int N_shard, int N_total, int L, int p, int token_major, void* dattn, cudaStream_t st) {
  Pyramid pyr; pyr.init(N_shard, L, p);
  if (!aligned16(dout) || !aligned16(dattn)) { set_error("scatter_bwd: pointers must be 16-byte aligned"); return LH_ERR_ARG; }
  int cs; uint32_t n;
  int rc = row_geometry("scatter_bwd", dtype, D, (long long)B * H * S_sel, &cs, &n);
  if (rc) return rc;
  FastDiv fs(S_sel);
  const long long row_stride = token_major ? (long long)H * D : D;
  const long long b_stride = (long long)H * N_total * D;
  const long long h_stride = token_major ? D : (long long)N_total * D;
  if (dtype == LH_DTYPE_BF16)
    scatter_bwd_kernel<__nv_bfloat16><<<grid_for(n), kRowThreads, 0, st>>>((const __nv_bfloat16*)dout, indices, pyr, log2i(p), D, fs, N_total, (__nv_bfloat16*)dattn, cs, n, H, row_stride, b_stride, h_stride);
  else
    scatter_bwd_kernel<float><<<grid_for(n), kRowThreads, 0, st>>>((const float*)dout, indices, pyr, log2i(p), D, fs, N_total, (float*)dattn, cs, n, H, row_stride, b_stride, h_stride);
  return check_launch("scatter_bwd_kernel");
}

int scatter_bwd(const void* dout, const int32_t* indices, int dtype, int B, int H, int S_sel, int D,
                int N_shard, int N_total, int L, int p, void* dattn, cudaStream_t st) {
  return scatter_bwd_layout(dout, indices, dtype, B, H, S_sel, D, N_shard, N_total, L, p, 0, dattn, st);
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
  const void* ptrs[] = {dq, dk, dv, dxq, dxk, dxv};
  for (const void* q : ptrs) if (q && !aligned16(q)) { set_error("unpool_bwd: pointers must be 16-byte aligned"); return LH_ERR_ARG; }
  int cs; uint32_t n;
  int rc = row_geometry("unpool_bwd", dtype, D, (long long)B * S * H, &cs, &n);
  if (rc) return rc;
  if (launch_grouped_rows<false>(dtype, L, cs, dq, dk, dv, dxq, dxk, dxv, 3, inverse, pyr, log2i(p), D, S_sel, S,
                                 B, H, (long long)H * D, (long long)S * H * D, D, st))
    return check_launch("unpool_bwd (grouped)");
  dim3 grid(grid_for(n), 3);
  FastDiv fh(H), fs(S);
  auto go = [&](auto lv) {
    constexpr int LV = decltype(lv)::value;
    if (dtype == LH_DTYPE_BF16) {
      using T = __nv_bfloat16;
      unpool_bwd_kernel<T, LV><<<grid, kRowThreads, 0, st>>>((const T*)dq, (const T*)dk, (const T*)dv, (T*)dxq, (T*)dxk, (T*)dxv, inverse, pyr, log2i(p), fh, fs, D, S_sel, cs, n);
    } else {
      using T = float;
      unpool_bwd_kernel<T, LV><<<grid, kRowThreads, 0, st>>>((const T*)dq, (const T*)dk, (const T*)dv, (T*)dxq, (T*)dxk, (T*)dxv, inverse, pyr, log2i(p), fh, fs, D, S_sel, cs, n);
    }
  };
  if (!dispatch_levels(L, go)) { set_error("unpool_bwd: L must be in [1, 7]"); return LH_ERR_SHAPE; }
  return check_launch("unpool_bwd");
}

}  // namespace lh
