// Causal attention forward over the selected sequence on tcgen05 / TMEM.
//
// Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True) on the
// gathered sequence (reference src/lighthouse_selection.py:815).
//
// One CTA per (pair of 128-row query tiles A and B, b*h), 384 threads,
// warp-specialised (warpgroup 0 gives registers to the softmax warpgroups
// with setmaxnreg: 56 + 2 x 224 per thread-slot = the 3 x 168 of the launch):
//   warp 0      TMA producer: Q_A and Q_B once, then K and V tiles through
//               two-stage rings shared by both query tiles (K one tile ahead)
//   warp 1      TMEM owner + MMA issuer (one elected lane):
//                 S_X = Q_X K_j^T  -> TMEM S_X   (SS MMA, both K-major, SW128)
//                 O_X += P_X V_j   -> TMEM O_X   (TS MMA: P read from TMEM,
//                                                 V as an MN-major SW128 operand)
//   warps 4..7  softmax for tile A, warps 8..11 softmax for tile B: each thread
//               owns one query row (= TMEM lane), reads S with tcgen05.ld,
//               keeps the running max / sum in registers and writes P (bf16)
//               back over its own S columns with tcgen05.st.
// The issue order PV_A(j), S_A(j+1), PV_B(j), S_B(j+1) keeps the tensor core
// busy with one tile while the other tile's softmax runs.  Because S_X(j+1)
// is issued after PV_X(j), its completion also means O_X is up to date, so a
// softmax warp may rescale O_X in TMEM right after S_X(j+1) arrives.  O is
// rescaled only when a row max grows by more than 2^8 (the stale max is
// consistent for numerator and denominator).
//
// TMEM columns: S_A 0..127, S_B 128..255, O_A 256..383, O_B 384..511.
// Every mbarrier wait is bounded; on timeout the CTA sets a status flag and leaves.
#include <cudaTypedefs.h>

#include "lh_common.cuh"
#include "sm100.cuh"

namespace lh {

using namespace sm100;

namespace fwd {
constexpr int kTile = 128;       // query rows and key rows per tile
constexpr int kD = 128;          // head dim
constexpr int kBox = 16384;      // one 128 x 64 bf16 TMA box (128-byte rows)
constexpr int kTileBytes = 2 * kBox;
constexpr int kNst = 2;          // K/V stages
constexpr int kThreads = 384;   // 3 warpgroups: {producer, MMA, 2 idle}, softmax A, softmax B
__host__ __device__ constexpr uint32_t col_s(int x) { return x ? 128u : 0u; }
__host__ __device__ constexpr uint32_t col_o(int x) { return x ? 384u : 256u; }
constexpr uint32_t kTmemCols = 512;
}  // namespace fwd

__device__ int g_attn_status;    // set to 1 when a bounded wait gave up

struct FwdSmem {
  uint64_t q_full;
  uint64_t k0_full, kv_full[fwd::kNst], k_empty[fwd::kNst], v_empty[fwd::kNst];   // kv_full[j%2]: K_{j+1} and V_j
  uint64_t s_full[2], p_ready[2], o_final[2];
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(fwd::kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, float* __restrict__ LSE,
                int S_q, int S_kv, int q_off, int n_pairs, float scale2) {
  using namespace fwd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;                                  // Q_A, Q_B
  uint8_t* sK = base + 2 * kTileBytes;
  uint8_t* sV = base + (2 + kNst) * kTileBytes;
  FwdSmem* sm = reinterpret_cast<FwdSmem*>(base + (2 + 2 * kNst) * kTileBytes);

  const int bh = blockIdx.x;
  const int pair = n_pairs - 1 - blockIdx.y;           // heaviest query tiles first
  const int n_qt = (S_q + kTile - 1) / kTile;
  const int n_kt = (S_kv + kTile - 1) / kTile;
  int qt[2], nkv[2], q_lo[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    qt[x] = 2 * pair + x;
    q_lo[x] = q_off + qt[x] * kTile;
    const int q_hi = q_off + min(qt[x] * kTile + kTile, S_q) - 1;
    nkv[x] = qt[x] < n_qt ? min(n_kt, q_hi / kTile + 1) : 0;   // causal: key tiles this tile sees
  }
  const int nkv_max = max(nkv[0], nkv[1]);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A CTA of an earlier launch gave up a wait: do nothing until the host resets.
  if (*reinterpret_cast<volatile int*>(&g_attn_status)) return;

  if (threadIdx.x == 0) {
    mbar_init(&sm->q_full, 1);
    for (int s = 0; s < kNst; ++s) { mbar_init(&sm->kv_full[s], 1); mbar_init(&sm->k_empty[s], 1); mbar_init(&sm->v_empty[s], 1); }
    mbar_init(&sm->k0_full, 1);
    for (int x = 0; x < 2; ++x) { mbar_init(&sm->s_full[x], 1); mbar_init(&sm->p_ready[x], 129); mbar_init(&sm->o_final[x], 1); }
    sm->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm->tmem_base;
  volatile int* abort = &sm->abort;

  if (warp < 4) {
  // Warpgroup 0 hands registers to the softmax warpgroups (one aligned setmaxnreg per warpgroup).
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmK); tma_prefetch_desc(&tmV);
      const bool two = nkv[1] > 0;
      mbar_expect_tx(&sm->q_full, (two ? 2 : 1) * kTileBytes);
      tma_load_3d(sQ, &tmQ, &sm->q_full, 0, qt[0] * kTile, bh);
      tma_load_3d(sQ + kBox, &tmQ, &sm->q_full, 64, qt[0] * kTile, bh);
      if (two) {
        tma_load_3d(sQ + kTileBytes, &tmQ, &sm->q_full, 0, qt[1] * kTile, bh);
        tma_load_3d(sQ + kTileBytes + kBox, &tmQ, &sm->q_full, 64, qt[1] * kTile, bh);
      }
    }
    // K runs one tile ahead of V: K_j is free once S(j) of both query tiles is
    // done (one step before V_j, which PV(j) reads), so its refill starts a
    // step earlier.  K_{j+1} and V_j share one barrier: the MMA warp waits once
    // per step for both (every wait of the issuing thread idles the pipe).
    auto load_k = [&](int j, uint64_t* bar) -> bool {
      const int st = j % kNst, round = j / kNst;
      if (round > 0 && !mbar_wait(&sm->k_empty[st], (round - 1) & 1, abort)) return false;
      if (lane == 0) {
        tma_load_3d(sK + st * kTileBytes, &tmK, bar, 0, j * kTile, bh);
        tma_load_3d(sK + st * kTileBytes + kBox, &tmK, bar, 64, j * kTile, bh);
      }
      return true;
    };
    bool ok = true;
    if (nkv_max > 0) {
      if (lane == 0) mbar_expect_tx(&sm->k0_full, kTileBytes);
      ok = load_k(0, &sm->k0_full);
    }
    for (int j = 0; j < nkv_max && ok; ++j) {
      const int st = j % kNst, round = j / kNst;
      const bool next_k = j + 1 < nkv_max;
      if (round > 0) ok = mbar_wait(&sm->v_empty[st], (round - 1) & 1, abort);
      if (__any_sync(0xffffffffu, !ok)) break;
      if (lane == 0) mbar_expect_tx(&sm->kv_full[st], (next_k ? 2 : 1) * kTileBytes);
      if (next_k) ok = load_k(j + 1, &sm->kv_full[st]);
      if (__any_sync(0xffffffffu, !ok)) break;
      if (lane == 0) {
        tma_load_3d(sV + st * kTileBytes, &tmV, &sm->kv_full[st], 0, j * kTile, bh);
        tma_load_3d(sV + st * kTileBytes + kBox, &tmV, &sm->kv_full[st], 64, j * kTile, bh);
      }
      __syncwarp();
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ K/V gate
    // Folds "V_j and K_{j+1} have landed" into p_ready of every tile active at
    // step j (129 = 128 softmax threads + this warp), so the MMA warp waits
    // only on p_ready: each wait of the issuing thread idles the tensor pipe.
    // A phase of p_ready gets this warp's arrival only after the previous one
    // has completed, so an early arrival never counts toward the wrong step.
    bool ok = true;
    for (int j = 0; j < nkv_max && ok; ++j) {
      ok = mbar_wait(&sm->kv_full[j % kNst], (j / kNst) & 1, abort);
      if (ok && lane == 0) {
        if (j < nkv[0]) mbar_arrive(&sm->p_ready[0]);
        if (j < nkv[1]) mbar_arrive(&sm->p_ready[1]);
      }
#pragma unroll
      for (int x = 0; x < 2; ++x)
        if (ok && j < (x ? nkv[1] : nkv[0])) ok = mbar_wait(&sm->p_ready[x], j & 1, abort);
      if (__any_sync(0xffffffffu, !ok)) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_bf16_f32(kTile, kTile, false, false);
    constexpr uint32_t idesc_pv = idesc_bf16_f32(kTile, kD, false, true);
    auto issue_s = [&](int x, int j) {
      const uint32_t q_addr = smem_u32(sQ + x * kTileBytes);
      const uint32_t k_addr = smem_u32(sK + (j % kNst) * kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
        mma_ss(tbase + col_s(x), smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024),
               idesc_qk, kk > 0);
      }
      mma_commit(&sm->s_full[x]);
    };
    auto issue_pv = [&](int x, int j, int nkv_x) {
      const uint32_t v_addr = smem_u32(sV + (j % kNst) * kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk)
        // 16 key rows per step: P columns advance by 8 (two bf16 per column),
        // V rows advance by 16 x 128 B; the two 64-wide d blocks sit kBox apart.
        mma_ts(tbase + col_o(x), tbase + col_s(x) + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kBox, 1024),
               idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
      if (j == nkv_x - 1) mma_commit(&sm->o_final[x]);
    };
    bool ok = mbar_wait(&sm->q_full, 0, abort) && mbar_wait(&sm->k0_full, 0, abort);
    if (!__any_sync(0xffffffffu, !ok)) {
      tc_fence_after();
      if (lane == 0) {
        issue_s(0, 0);
        if (nkv[1] > 0) issue_s(1, 0);
        mma_commit(&sm->k_empty[0]);              // K_0 no longer read once these complete
      }
      __syncwarp();
      for (int j = 0; j < nkv_max && ok; ++j) {
        const int st = j % kNst;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const int nkv_x = x ? nkv[1] : nkv[0];
          if (j >= nkv_x) continue;
          ok = mbar_wait(&sm->p_ready[x], j & 1, abort);
          if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
          tc_fence_after();
          if (lane == 0) {
            issue_pv(x, j, nkv_x);
            if (j + 1 < nkv_x) issue_s(x, j + 1);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) {
          mma_commit(&sm->v_empty[st]);                           // V_j read by PV(j) of both tiles
          if (j + 1 < nkv_max) mma_commit(&sm->k_empty[(j + 1) % kNst]);   // K_{j+1} read by S(j+1)
        }
        __syncwarp();
      }
    }
  }
  } else {
    // ------------------------------------------------------------ softmax (tile A: warps 4-7, B: 8-11)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
    const int x = warp < 8 ? 0 : 1;
    const int my_qt = x ? qt[1] : qt[0];
    const int my_nkv = x ? nkv[1] : nkv[0];
    const int my_qlo = x ? q_lo[1] : q_lo[0];
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qrow = my_qt * kTile + row;        // row inside this (b,h) slice of Q
    const int qpos = q_off + qrow;               // global causal position
    const uint32_t lane_base = tbase + ((uint32_t)(quad * 32) << 16);
    const uint32_t s_col = col_s(x), o_col = col_o(x);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < my_nkv; ++j) {
      ok = mbar_wait(&sm->s_full[x], j & 1, abort);
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_base + s_col + c * 32, s[c]);
      tmem_ld_wait();
      const bool need_mask = (j * kTile + kTile - 1 > my_qlo) || (j * kTile + kTile > S_kv);
      // eight independent partial maxima instead of one 128-long dependency chain
      float mxp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mxp[u] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (need_mask) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int kvpos = j * kTile + c * 32 + e;
            if (kvpos > qpos || kvpos >= S_kv) s[c][e] = __float_as_uint(-INFINITY);
          }
        }
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          mxp[(e >> 1) & 7] = fmax3(mxp[(e >> 1) & 7], __uint_as_float(s[c][e]), __uint_as_float(s[c][e + 1]));
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                             fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      const float mx2 = mx * scale2;
      if (j == 0) {
        m = mx2;
      } else if (__any_sync(0xffffffffu, mx2 > m + 8.0f)) {
        // O_X already holds PV_X(j-1): S_X(j) was issued after it.
        const float mnew = fmaxf(m, mx2);
        const float alpha = ex2(m - mnew);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_base + o_col + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(lane_base + o_col + c * 32, o);
        }
        l *= alpha;
        m = mnew;
      }
      // exponent arguments and row sums two lanes at a time (fma.rn.f32x2 / add.rn.f32x2)
      float2 rsp[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) rsp[u] = make_float2(0.f, 0.f);
      const float2 sc2 = make_float2(scale2, scale2), negm = make_float2(-m, -m);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int i0 = h * 64 + 2 * e;
          const float2 sv = make_float2(__uint_as_float(s[i0 >> 5][i0 & 31]),
                                        __uint_as_float(s[(i0 + 1) >> 5][(i0 + 1) & 31]));
          const float2 arg = ffma2(sv, sc2, negm);
          const float2 pv = make_float2(ex2(arg.x), ex2(arg.y));
          rsp[e & 3] = fadd2(rsp[e & 3], pv);
          pk[e] = pack_bf16(pv.x, pv.y);
        }
        tmem_st32(lane_base + s_col + h * 32, pk);
      }
      const float2 r01 = fadd2(rsp[0], rsp[1]), r23 = fadd2(rsp[2], rsp[3]);
      const float2 r = fadd2(r01, r23);
      const float rs = r.x + r.y;
      tmem_st_wait();
      l += rs;
      tc_fence_before();
      mbar_arrive(&sm->p_ready[x]);
    }
    if (ok && my_nkv > 0) ok = mbar_wait(&sm->o_final[x], 0, abort);
    if (my_nkv > 0 && !__any_sync(0xffffffffu, !ok)) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      __nv_bfloat16* orow = O + ((size_t)bh * S_q + qrow) * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + o_col + c * 32, o);
        tmem_ld_wait();
        if (qrow < S_q) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[v4 * 8 + 0]) * inv_l, __uint_as_float(o[v4 * 8 + 1]) * inv_l);
            w.y = pack_bf16(__uint_as_float(o[v4 * 8 + 2]) * inv_l, __uint_as_float(o[v4 * 8 + 3]) * inv_l);
            w.z = pack_bf16(__uint_as_float(o[v4 * 8 + 4]) * inv_l, __uint_as_float(o[v4 * 8 + 5]) * inv_l);
            w.w = pack_bf16(__uint_as_float(o[v4 * 8 + 6]) * inv_l, __uint_as_float(o[v4 * 8 + 7]) * inv_l);
            *reinterpret_cast<uint4*>(orow + c * 32 + v4 * 8) = w;
          }
        }
      }
      if (qrow < S_q) LSE[(size_t)bh * S_q + qrow] = (m + __log2f(l)) * 0.69314718055994531f;
    }
  }


  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
  if (threadIdx.x == 0 && sm->abort) atomicExch(&g_attn_status, 1);
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// (BH, rows, 128) bf16 tensor viewed as 3-D {128, rows, BH}; boxes of
// 64 columns x box_rows rows with the 128-byte swizzle.
int make_tmap_rows(CUtensorMap* m, const void* ptr, int rows, int BH, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return LH_ERR_LAUNCH; }
  if ((uintptr_t)ptr & 15) { set_error("attention operands must be 16-byte aligned"); return LH_ERR_ARG; }
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)BH};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)rows * 128 * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return LH_ERR_LAUNCH; }
  return LH_OK;
}

// (BH, rows, 128) fp32 tensor viewed as 3-D {128, rows, BH}; boxes of 32
// columns (128 bytes) x 128 rows with the 128-byte swizzle (dQ accumulator).
int make_tmap_rows_f32(CUtensorMap* m, const void* ptr, int rows, int BH) {
  auto enc = get_encode_fn();
  if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return LH_ERR_LAUNCH; }
  if ((uintptr_t)ptr & 15) { set_error("dQ accumulator must be 16-byte aligned"); return LH_ERR_ARG; }
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)BH};
  cuuint64_t strides[2] = {128 * 4, (cuuint64_t)rows * 128 * 4};
  cuuint32_t box[3] = {32, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled (f32) failed (%d)", (int)r); return LH_ERR_LAUNCH; }
  return LH_OK;
}

int attn_fwd(const void* q, const void* k, const void* v, int B, int H, int S_q, int S_kv, int q_off, int D,
             float scale, void* o, float* lse, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_tmap_rows(&mq, q, S_q, B * H, 128))) return rc;
  if ((rc = make_tmap_rows(&mk, k, S_kv, B * H, 128))) return rc;
  if ((rc = make_tmap_rows(&mv, v, S_kv, B * H, 128))) return rc;
  const int n_qt = (S_q + fwd::kTile - 1) / fwd::kTile;
  const int n_pairs = (n_qt + 1) / 2;
  const size_t smem = 1024 + fwd::kTileBytes * (2 + 2 * fwd::kNst) + sizeof(FwdSmem);
  cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(B * H, n_pairs);
  attn_fwd_kernel<<<grid, fwd::kThreads, smem, st>>>(mq, mk, mv, (__nv_bfloat16*)o, lse, S_q, S_kv, q_off, n_pairs,
                                                    scale * 1.4426950408889634f);
  return check_launch("attn_fwd_kernel");
}

// Merge of two partial attentions of the same queries over disjoint key
// sets (log-sum-exp combination): with m = max(lse1, lse2),
//   lse = m + log(e^(lse1-m) + e^(lse2-m)),
//   o   = (e^(lse1-lse) o1 + e^(lse2-lse) o2).
// One warp per query row, four head-dimension elements per lane.
__global__ void attn_merge_kernel(const __nv_bfloat16* __restrict__ o1, const float* __restrict__ lse1,
                                  const __nv_bfloat16* __restrict__ o2, const float* __restrict__ lse2,
                                  __nv_bfloat16* __restrict__ o, float* __restrict__ lse, long long rows) {
  const long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float a = lse1[r], b = lse2[r];
  const float m = fmaxf(a, b);
  float w1 = 0.f, w2 = 0.f, l = m;
  if (m != -INFINITY) {
    const float e1 = __expf(a - m), e2 = __expf(b - m);
    l = m + __logf(e1 + e2);
    w1 = __expf(a - l);
    w2 = __expf(b - l);
  }
  const size_t off = (size_t)r * 128 + lane * 4;
  const uint2 x = *reinterpret_cast<const uint2*>(o1 + off);
  const uint2 y = *reinterpret_cast<const uint2*>(o2 + off);
  const float2 x0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
  const float2 x1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
  const float2 y0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&y.x));
  const float2 y1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&y.y));
  uint2 z;
  z.x = pack_bf16(w1 * x0.x + w2 * y0.x, w1 * x0.y + w2 * y0.y);
  z.y = pack_bf16(w1 * x1.x + w2 * y1.x, w1 * x1.y + w2 * y1.y);
  *reinterpret_cast<uint2*>(o + off) = z;
  if (lane == 0) lse[r] = l;
}

int attn_merge(const void* o1, const float* lse1, const void* o2, const float* lse2, long long rows, int D,
               void* o, float* lse, cudaStream_t st) {
  (void)D;
  const long long threads = rows * 32;
  attn_merge_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      (const __nv_bfloat16*)o1, lse1, (const __nv_bfloat16*)o2, lse2, (__nv_bfloat16*)o, lse, rows);
  return check_launch("attn_merge_kernel");
}

int attn_bwd_status(int reset);

int attn_status(int reset) {
  int h = attn_bwd_status(reset);
  int f = 0;
  cudaMemcpyFromSymbol(&f, g_attn_status, sizeof(int));
  h |= f;
  if (reset) { int z = 0; cudaMemcpyToSymbol(g_attn_status, &z, sizeof(int)); }
  return h;
}

}  // namespace lh
