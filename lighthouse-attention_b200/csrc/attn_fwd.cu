// Causal attention forward over the selected sequence on tcgen05 / TMEM.
//
// Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True) on the
// gathered sequence (reference src/lighthouse_selection.py:815).
//
// One CTA per (128-row query tile, b*h), 192 threads, warp-specialised:
//   warp 0      TMA producer: Q once, then K/V tiles through an NST-stage ring
//   warp 1      TMEM owner + MMA issuer (one elected lane):
//                 S_j = Q K_j^T  -> TMEM S[j%2]  (SS MMA, both K-major, SW128)
//                 O  += P_j V_j  -> TMEM O       (TS MMA: P read from TMEM,
//                                                 V as an MN-major SW128 operand)
//   warps 2..5  softmax: each thread owns one query row (= TMEM lane), reads
//               S with tcgen05.ld, keeps the running max / sum in registers,
//               writes P (bf16) back over its own S columns with tcgen05.st.
//               O is rescaled in TMEM only when a row max grows by more than
//               2^8 (the stale max is consistent for numerator and
//               denominator, so the result is exact up to rounding).
// S_{j+1} is issued before PV_j so that the tensor core works on the next
// tile while the softmax warps handle the current one.
//
// TMEM columns: S[0] 0..127, S[1] 128..255, O 256..383 (512 allocated).
// Every mbarrier wait is bounded; on timeout the CTA sets *status and leaves.
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
constexpr int kThreads = 192;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256, kTmemCols = 512;
}  // namespace fwd

__device__ int g_attn_status;    // set to 1 when a bounded wait gave up

template <int NST>
struct FwdSmem {
  uint64_t q_full, o_final;
  uint64_t k_full[NST], v_full[NST], kv_empty[NST];
  uint64_t s_full[2], p_full[2], o_done;
  uint32_t tmem_base;
  int abort;
};

template <int NST>
__global__ void __launch_bounds__(fwd::kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O, float* __restrict__ LSE,
                int S_q, int S_kv, int q_off, int n_qt, float scale2) {
  using namespace fwd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK = base + kTileBytes;
  uint8_t* sV = base + kTileBytes * (1 + NST);
  FwdSmem<NST>* sm = reinterpret_cast<FwdSmem<NST>*>(base + kTileBytes * (1 + 2 * NST));

  const int bh = blockIdx.x;
  const int qt = n_qt - 1 - blockIdx.y;      // heaviest query tiles first
  // Causal over global positions: query row r sits at q_off + r, key row c at c.
  const int q_lo = q_off + qt * kTile;
  const int q_hi = q_off + min(qt * kTile + kTile, S_q) - 1;
  const int nkv = min((S_kv + kTile - 1) / kTile, q_hi / kTile + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A CTA of an earlier launch gave up a wait: do nothing until the host resets.
  if (*reinterpret_cast<volatile int*>(&g_attn_status)) return;

  if (threadIdx.x == 0) {
    mbar_init(&sm->q_full, 1);
    mbar_init(&sm->o_final, 1);
    for (int s = 0; s < NST; ++s) { mbar_init(&sm->k_full[s], 1); mbar_init(&sm->v_full[s], 1); mbar_init(&sm->kv_empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&sm->s_full[b], 1); mbar_init(&sm->p_full[b], 128); }
    mbar_init(&sm->o_done, 1);
    sm->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm->tmem_base;
  volatile int* abort = &sm->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ); tma_prefetch_desc(&tmK); tma_prefetch_desc(&tmV);
      mbar_expect_tx(&sm->q_full, kTileBytes);
      tma_load_3d(sQ, &tmQ, &sm->q_full, 0, qt * kTile, bh);
      tma_load_3d(sQ + kBox, &tmQ, &sm->q_full, 64, qt * kTile, bh);
    }
    for (int j = 0; j < nkv; ++j) {
      const int st = j % NST, round = j / NST;
      if (round > 0) {
        bool ok = mbar_wait(&sm->kv_empty[st], (round - 1) & 1, abort);
        if (__any_sync(0xffffffffu, !ok)) break;
      }
      if (lane == 0) {
        mbar_expect_tx(&sm->k_full[st], kTileBytes);
        tma_load_3d(sK + st * kTileBytes, &tmK, &sm->k_full[st], 0, j * kTile, bh);
        tma_load_3d(sK + st * kTileBytes + kBox, &tmK, &sm->k_full[st], 64, j * kTile, bh);
        mbar_expect_tx(&sm->v_full[st], kTileBytes);
        tma_load_3d(sV + st * kTileBytes, &tmV, &sm->v_full[st], 0, j * kTile, bh);
        tma_load_3d(sV + st * kTileBytes + kBox, &tmV, &sm->v_full[st], 64, j * kTile, bh);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_bf16_f32(kTile, kTile, false, false);
    constexpr uint32_t idesc_pv = idesc_bf16_f32(kTile, kD, false, true);
    const uint32_t q_addr = smem_u32(sQ);
    auto issue_s = [&](int j) {
      const int st = j % NST;
      const uint32_t k_addr = smem_u32(sK + st * kTileBytes);
      const uint32_t d_tmem = tbase + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
        mma_ss(d_tmem, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024), idesc_qk,
               kk > 0);
      }
      mma_commit(&sm->s_full[j & 1]);
    };
    bool ok = mbar_wait(&sm->q_full, 0, abort);
    ok = ok && mbar_wait(&sm->k_full[0], 0, abort);
    if (!__any_sync(0xffffffffu, !ok)) {
      tc_fence_after();
      if (lane == 0) issue_s(0);
      __syncwarp();
      for (int j = 0; j < nkv; ++j) {
        if (j + 1 < nkv) {
          ok = mbar_wait(&sm->k_full[(j + 1) % NST], ((j + 1) / NST) & 1, abort);
          if (__any_sync(0xffffffffu, !ok)) break;
          tc_fence_after();
          if (lane == 0) issue_s(j + 1);
          __syncwarp();
        }
        const int st = j % NST;
        ok = mbar_wait(&sm->v_full[st], (j / NST) & 1, abort);
        ok = ok && mbar_wait(&sm->p_full[j & 1], (j >> 1) & 1, abort);
        if (__any_sync(0xffffffffu, !ok)) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t v_addr = smem_u32(sV + st * kTileBytes);
          const uint32_t p_tmem = tbase + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < kTile / 16; ++kk) {
            // 16 key rows per step: P columns advance by 8 (two bf16 per column),
            // V rows advance by 16 x 128 B; the two 64-wide d blocks sit kBox apart.
            mma_ts(tbase + kColO, p_tmem + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kBox, 1024), idesc_pv,
                   (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&sm->o_done);
          mma_commit(&sm->kv_empty[st]);
          if (j == nkv - 1) mma_commit(&sm->o_final);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qrow = qt * kTile + row;          // row inside this (b,h) slice of Q
    const int qpos = q_off + qrow;              // global causal position
    const uint32_t lane_base = tbase + ((uint32_t)(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int b = j & 1;
      const uint32_t s_col = b ? kColS1 : kColS0;
      ok = mbar_wait(&sm->s_full[b], (j >> 1) & 1, abort);
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_base + s_col + c * 32, s[c]);
      tmem_ld_wait();
      const bool need_mask = (j * kTile + kTile - 1 > q_lo) || (j * kTile + kTile > S_kv);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float v = __uint_as_float(s[c][e]);
          const int kvpos = j * kTile + c * 32 + e;
          if (need_mask && (kvpos > qpos || kvpos >= S_kv)) { v = -INFINITY; s[c][e] = __float_as_uint(v); }
          mx = fmaxf(mx, v);
        }
      }
      const float mx2 = mx * scale2;
      if (j == 0) {
        m = mx2;
      } else if (__any_sync(0xffffffffu, mx2 > m + 8.0f)) {
        const float mnew = fmaxf(m, mx2);
        const float alpha = ex2(m - mnew);
        ok = mbar_wait(&sm->o_done, (j - 1) & 1, abort);
        if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_base + kColO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(lane_base + kColO + c * 32, o);
        }
        tmem_st_wait();
        l *= alpha;
        m = mnew;
      }
      float rs = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int i0 = h * 64 + 2 * e;
          const float p0 = ex2(fmaf(__uint_as_float(s[i0 >> 5][i0 & 31]), scale2, -m));
          const float p1 = ex2(fmaf(__uint_as_float(s[(i0 + 1) >> 5][(i0 + 1) & 31]), scale2, -m));
          rs += p0 + p1;
          pk[e] = pack_bf16(p0, p1);
        }
        tmem_st32(lane_base + s_col + h * 32, pk);
      }
      tmem_st_wait();
      l += rs;
      tc_fence_before();
      mbar_arrive(&sm->p_full[b]);
    }
    if (ok) ok = mbar_wait(&sm->o_final, 0, abort);
    if (!__any_sync(0xffffffffu, !ok)) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      __nv_bfloat16* orow = O + ((size_t)bh * S_q + qrow) * kD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + kColO + c * 32, o);
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
// 64 columns x 128 rows with the 128-byte swizzle.
int make_tmap_rows(CUtensorMap* m, const void* ptr, int rows, int BH) {
  auto enc = get_encode_fn();
  if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return LH_ERR_LAUNCH; }
  if ((uintptr_t)ptr & 15) { set_error("attention operands must be 16-byte aligned"); return LH_ERR_ARG; }
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)BH};
  cuuint64_t strides[2] = {128 * 2, (cuuint64_t)rows * 128 * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return LH_ERR_LAUNCH; }
  return LH_OK;
}

int attn_fwd(const void* q, const void* k, const void* v, int B, int H, int S_q, int S_kv, int q_off, int D,
             float scale, void* o, float* lse, cudaStream_t st) {
  constexpr int NST = 2;
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_tmap_rows(&mq, q, S_q, B * H))) return rc;
  if ((rc = make_tmap_rows(&mk, k, S_kv, B * H))) return rc;
  if ((rc = make_tmap_rows(&mv, v, S_kv, B * H))) return rc;
  const int n_qt = (S_q + fwd::kTile - 1) / fwd::kTile;
  const size_t smem = 1024 + fwd::kTileBytes * (1 + 2 * NST) + sizeof(FwdSmem<NST>);
  auto kern = attn_fwd_kernel<NST>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(B * H, n_qt);
  kern<<<grid, fwd::kThreads, smem, st>>>(mq, mk, mv, (__nv_bfloat16*)o, lse, S_q, S_kv, q_off, n_qt,
                                           scale * 1.4426950408889634f);
  return check_launch("attn_fwd_kernel");
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
