// Causal attention backward on tcgen05 / TMEM (dQ, dK, dV).
//
// Backward of F.scaled_dot_product_attention(is_causal=True) on the selected
// sequence (reference src/lighthouse_selection.py:815), with the same causal
// geometry as attn_fwd.cu (query row r at position q_off + r, key row c at c).
//
// Three launches:
//   1. prep:  Delta[q] = sum_d dO[q,d] * O[q,d] (fp32), dQacc = 0
//   2. main:  one CTA per (128-key tile j, b*h); K_j and V_j stay in shared
//             memory while the CTA walks every query tile i that can see them.
//             Each query tile is handled as two 64-query halves h so that the
//             elementwise work on one half overlaps the MMAs of the other:
//               S^T_h  = K_j Q_h^T            (SS, N = 64, TMEM cols  64h..)
//               dP^T_h = V_j dO_h^T           (SS, N = 64, TMEM cols 128 + 64h..)
//             compute warps (one key row per thread = TMEM lane, 32 queries each):
//               P^T  = exp2(S^T * scale*log2e - lse2[q])
//               dS^T = P^T * (dP^T - Delta[q])
//             both as bf16 pairs back into the warp's own S^T columns, and dS^T
//             also into shared memory;
//               dV_j += P^T_h dO_h            (TS, TMEM cols 256..383)
//               dK_j += dS^T_h Q_h            (TS, TMEM cols 384..511)
//               dQ_h^T = K_j^T dS_h^T         (SS, both MN-major, N = 64, issued per
//                                              half into the dP^T_h columns 128 + 64h..)
//             a drain warpgroup reads dQ_h^T (TMEM lane = head dimension) and
//             adds it into the fp32 dQacc with coalesced red.global.add: no
//             shared-memory stage, so shared-memory bandwidth (which the SS
//             MMAs saturate) is left to the MMAs and the Q / dO refills, and the
//             freed 64 KB double-buffers Q_i / dO_i.  At the end dK (times
//             scale) and dV are written as bf16.
//   3. post:  dQ = bf16(dQacc * scale)
// Shared-memory operands use the 128-byte swizzle; Q_i / dO_i / K_j / V_j
// arrive by TMA (no multicast).  Every mbarrier wait is bounded.
#include <cudaTypedefs.h>

#include <mutex>

#include "lh_common.cuh"
#include "sm100.cuh"

namespace lh {

using namespace sm100;

__device__ int g_attn_bwd_status;   // set to 1 when a bounded wait gave up
int make_tmap_rows(CUtensorMap* m, const void* ptr, int rows, int BH, int box_rows);

namespace bwd {
constexpr int kTile = 128;
constexpr int kD = 128;
constexpr int kBox = 16384;
constexpr int kTileBytes = 2 * kBox;
// warpgroup 0: {TMA producer, MMA issuer, 2 idle}; warpgroup 1: dQ drain;
// warpgroups 2-5: P / dS (four warps per TMEM lane quadrant, 16 queries of each half)
constexpr int kThreads = 768;
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384, kTmemCols = 512;
constexpr int kStages = 2;                 // Q_i / dO_i buffers
}  // namespace bwd

struct BwdSmem {
  uint64_t kv_full, mma_done;
  uint64_t dq_ready[2];                                          // dQ^T of query half h complete
  uint64_t dq_free[2];                                           // dQ^T query columns [64h, 64h+64) read
  uint64_t q_full[bwd::kStages][2], q_empty[bwd::kStages][2];   // per stage and 64-query half
  uint64_t s_ready[2], p_ready[2];                               // per 64-query half
  uint32_t tmem_base;
  int abort;
  __align__(16) float lse2[2][bwd::kTile];     // read as float4
  __align__(16) float delta[2][bwd::kTile];
};
static_assert(offsetof(BwdSmem, lse2) % 16 == 0 && offsetof(BwdSmem, delta) % 16 == 0, "float4 reads");
static_assert((3 + 2 * bwd::kStages) * bwd::kTileBytes + sizeof(BwdSmem) <= 232448, "shared memory per CTA");

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// 16-byte store of 8 bf16 into the SW128 K-major layout of a 128 x 128 tile
// stored as two 64-column boxes: row r, columns [8c, 8c+8).
__device__ __forceinline__ void st_sw128(uint8_t* tile, int r, int c, uint4 v) {
  const int box = c >> 3, chunk = c & 7;
  *reinterpret_cast<uint4*>(tile + box * bwd::kBox + r * 128 + ((chunk ^ (r & 7)) << 4)) = v;
}

__global__ void __launch_bounds__(bwd::kThreads, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                const float* __restrict__ LSE, const float* __restrict__ Delta, float* __restrict__ dQacc,
                __nv_bfloat16* __restrict__ dK, __nv_bfloat16* __restrict__ dV, int S_q, int S_kv, int q_off,
                float scale2, float scale) {
  using namespace bwd;
  // 7 bf16 tiles + barriers fill 227 KB: no room for alignment slack, so the
  // dynamic window itself must be 1024-byte aligned.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw;
  uint8_t* sK = base;
  uint8_t* sV = base + kTileBytes;
  uint8_t* sQ = base + 2 * kTileBytes;                  // kStages tiles
  uint8_t* sdO = base + (2 + kStages) * kTileBytes;     // kStages tiles
  uint8_t* sdS = base + (2 + 2 * kStages) * kTileBytes;
  BwdSmem* sm = reinterpret_cast<BwdSmem*>(base + (3 + 2 * kStages) * kTileBytes);

  const int bh = blockIdx.x;
  const int j = blockIdx.y;                      // key tile (heaviest first: j = 0 sees every query)
  const int n_qt = (S_q + kTile - 1) / kTile;
  int i0 = (j * kTile - q_off) / kTile;          // first query tile with a row at position >= j*128
  if (j * kTile - q_off < 0) i0 = 0;
  const int n_it = n_qt - i0 > 0 ? n_qt - i0 : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (*reinterpret_cast<volatile int*>(&g_attn_bwd_status)) return;
  if (smem_u32(smem_raw) & 1023u) {               // layout assumption broken: report instead of corrupting
    if (threadIdx.x == 0) atomicExch(&g_attn_bwd_status, 1);
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(&sm->kv_full, 1);
    mbar_init(&sm->mma_done, 1);
    for (int h = 0; h < 2; ++h) {
      mbar_init(&sm->dq_ready[h], 1);
      for (int s = 0; s < kStages; ++s) {
        mbar_init(&sm->q_full[s][h], 1);
        mbar_init(&sm->q_empty[s][h], 1);
      }
      mbar_init(&sm->s_ready[h], 1);
      mbar_init(&sm->p_ready[h], 512);
      mbar_init(&sm->dq_free[h], 128);
    }
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
    // Register split 112 (this warpgroup) + 80 (drain) + 4 x 72 (P / dS) per
    // thread-slot equals the 6 x 80 of the launch (one aligned setmaxnreg per
    // warpgroup; .inc may not go below the launch's 80, .dec not above it).
    asm volatile("setmaxnreg.inc.sync.aligned.u32 112;\n" ::: "memory");
    if (warp == 0) {
      // ---------------------------------------------------------- TMA producer
      if (lane == 0 && n_it > 0) {
        mbar_expect_tx(&sm->kv_full, 2 * kTileBytes);
        tma_load_3d(sK, &tmK, &sm->kv_full, 0, j * kTile, bh);
        tma_load_3d(sK + kBox, &tmK, &sm->kv_full, 64, j * kTile, bh);
        tma_load_3d(sV, &tmV, &sm->kv_full, 0, j * kTile, bh);
        tma_load_3d(sV + kBox, &tmV, &sm->kv_full, 64, j * kTile, bh);
      }
      // Q_i and dO_i arrive in two 64-row halves into a ring of kStages tiles;
      // each half is refilled once the dV / dK MMAs of that half have read it.
      bool ok = true;
      for (int t = 0; t < n_it && ok; ++t) {
        const int i = i0 + t, st = t % kStages;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (t >= kStages) ok = mbar_wait(&sm->q_empty[st][h], ((t / kStages) - 1) & 1, abort);
          if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
          if (lane == 0) {
            const int row = i * kTile + h * 64;
            uint8_t* q = sQ + st * kTileBytes + h * (kBox / 2);
            uint8_t* d = sdO + st * kTileBytes + h * (kBox / 2);
            mbar_expect_tx(&sm->q_full[st][h], kTileBytes);
            tma_load_3d(q, &tmQ, &sm->q_full[st][h], 0, row, bh);
            tma_load_3d(q + kBox, &tmQ, &sm->q_full[st][h], 64, row, bh);
            tma_load_3d(d, &tmdO, &sm->q_full[st][h], 0, row, bh);
            tma_load_3d(d + kBox, &tmdO, &sm->q_full[st][h], 64, row, bh);
          }
          __syncwarp();
        }
      }
    } else if (warp == 1 || warp == 2) {
      // ---------------------------------------------------------- MMA issuers
      // Two issuing warps so that the tensor pipe stays fed while one of them
      // waits: its instruction queue is shallow, and a wait of the issuing
      // thread (even on a barrier that has already completed) leaves the pipe
      // idle for a shared-memory round trip.  Warp 1 issues S^T / dP^T, warp 2
      // dV / dK and dQ^T.  tcgen05.commit tracks the committing thread's own
      // MMAs, and every TMEM / shared-memory hazard between the two warps is
      // covered by a barrier below.
      constexpr uint32_t id_s = idesc_bf16_f32(kTile, 64, false, false);     // S^T / dP^T halves: N = 64 queries
      constexpr uint32_t id_kmn = idesc_bf16_f32(kTile, kD, false, true);    // A K-major (TMEM), B MN-major
      constexpr uint32_t id_mnmn = idesc_bf16_f32(kD, 64, true, true);       // dQ^T half: A MN-major, B MN-major
      // Descriptors are a per-operand base plus a constant offset (the start
      // address field holds addr >> 4 in its low 14 bits and every shared
      // address is below 256 KB, so the add cannot carry out of the field).
      // The empty asm keeps the compiler from hoisting every per-k descriptor
      // out of the tile loop, which would not fit this warpgroup's registers.
      auto kdesc = [](uint32_t addr) {            // K-major: lbo 16, sbo 1024
        uint64_t d = smem_desc_sw128(addr, 16, 1024);
        asm volatile("" : "+l"(d));
        return d;
      };
      auto mdesc = [](uint32_t addr) {            // MN-major: lbo = box stride, sbo 1024
        uint64_t d = smem_desc_sw128(addr, kBox, 1024);
        asm volatile("" : "+l"(d));
        return d;
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        const bool ok = mbar_wait(bar, parity, abort);
        if (__any_sync(0xffffffffu, !ok)) return false;
        tc_fence_after();
        return true;
      };
      bool ok = true;
      if (warp == 1) {
        // S^T_h and dP^T_h of tile t.  S^T_h overwrites P^T_h / dS^T_h of tile
        // t-1 (read by warp 2's dV / dK MMAs, complete when q_empty of that
        // half commits); dP^T_h overwrites half h of dQ^T of tile t-1 (read by
        // the drain warps, dq_free[h]).
        const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
        ok = n_it > 0 ? wait(&sm->kv_full, 0) : true;
        for (int t = 0; t < n_it && ok; ++t) {
          const int st = t % kStages;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            ok = wait(&sm->q_full[st][h], (t / kStages) & 1);
            if (ok && t > 0) ok = wait(&sm->q_empty[(t - 1) % kStages][h], ((t - 1) / kStages) & 1);
            if (!ok) break;
            if (lane == 0) {
              const uint64_t da = kdesc(aK), db = kdesc(smem_u32(sQ + st * kTileBytes) + h * (kBox / 2));
#pragma unroll
              for (int kk = 0; kk < kD / 16; ++kk) {
                const uint32_t off = ((kk >> 2) * kBox + (kk & 3) * 32) >> 4;
                mma_ss(tbase + kColS + h * 64, da + off, db + off, id_s, kk > 0);
              }
            }
            __syncwarp();
            if (t > 0) ok = wait(&sm->dq_free[h], (t - 1) & 1);
            if (!ok) break;
            if (lane == 0) {
              const uint64_t da = kdesc(aV), db = kdesc(smem_u32(sdO + st * kTileBytes) + h * (kBox / 2));
#pragma unroll
              for (int kk = 0; kk < kD / 16; ++kk) {
                const uint32_t off = ((kk >> 2) * kBox + (kk & 3) * 32) >> 4;
                mma_ss(tbase + kColDP + h * 64, da + off, db + off, id_s, kk > 0);
              }
              mma_commit(&sm->s_ready[h]);
            }
            __syncwarp();
          }
        }
      } else {
        // Per 64-query half h: dQ_h^T = K^T dS^T_h (into the dP^T_h columns,
        // which the compute warps have read), then dV += P^T_h dO_h and
        // dK += dS^T_h Q_h with A operands from TMEM: compute warp w of a
        // quadrant leaves the bf16 pairs of its 16 queries of half h at columns
        // [64h + 16w, +8) (P^T) and [64h + 16w + 8, +8) (dS^T).  Issuing dQ per
        // half lets the drain of half h, and with it the next tile's dP^T_h,
        // proceed while the compute warps work on the other half.
        const uint32_t aK = smem_u32(sK), adS = smem_u32(sdS);
        for (int t = 0; t < n_it && ok; ++t) {
          const int st = t % kStages;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            ok = wait(&sm->p_ready[h], t & 1);
            if (!ok) break;
            if (lane == 0) {
              {
                const uint64_t da = mdesc(aK), db = mdesc(adS + h * kBox);   // dS^T queries of half h: box h
#pragma unroll
                for (int kk = 0; kk < kTile / 16; ++kk)    // K = 16 key rows per step
                  mma_ss(tbase + kColDP + h * 64, da + ((kk * 2048) >> 4), db + ((kk * 2048) >> 4), id_mnmn,
                         kk > 0);
                mma_commit(&sm->dq_ready[h]);
              }
              const uint64_t dq = mdesc(smem_u32(sQ + st * kTileBytes) + h * 4 * 2048);
              const uint64_t ddo = mdesc(smem_u32(sdO + st * kTileBytes) + h * 4 * 2048);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t a = tbase + kColS + h * 64 + kk * 16;   // warp kk's 16 queries: P^T | dS^T
                const uint32_t acc = (t > 0 || h > 0 || kk > 0) ? 1u : 0u;
                mma_ts(tbase + kColDV, a, ddo + ((kk * 2048) >> 4), id_kmn, acc);
                mma_ts(tbase + kColDK, a + 8, dq + ((kk * 2048) >> 4), id_kmn, acc);
              }
              mma_commit(&sm->q_empty[st][h]);   // Q_h / dO_h of this stage and P^T_h / dS^T_h no longer read
            }
            __syncwarp();
          }
        }
        if (lane == 0) mma_commit(&sm->mma_done);   // every dV / dK MMA of this CTA has completed
        __syncwarp();
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ dQ drain (launch registers: 80)
    // TMEM lane = head-dimension column d; each thread adds its d of all 128
    // query rows: a warp's red.global.add covers one 128-byte row segment.
    const int quad = warp & 3;
    const int d = quad * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(quad * 32) << 16);
    bool ok = true;
    for (int t = 0; t < n_it && ok; ++t) {
      const int i = i0 + t;
      float* dst = dQacc + ((size_t)bh * S_q + (size_t)i * kTile) * kD + d;
      const int rows = S_q - i * kTile < kTile ? S_q - i * kTile : kTile;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {               // query rows [64h, 64h+64)
        ok = mbar_wait(&sm->dq_ready[h], t & 1, abort);
        if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
        tc_fence_after();
        uint32_t v[2][32];
        tmem_ld32(lane_base + kColDP + h * 64, v[0]);
        tmem_ld32(lane_base + kColDP + h * 64 + 32, v[1]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&sm->dq_free[h]);             // the MMA warp may overwrite these columns now
        float* p = dst + (size_t)(h * 64) * kD;
        if (rows == kTile) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) red_add_f32(p + (size_t)(c * 32 + e) * kD, __uint_as_float(v[c][e]));
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (h * 64 + c * 32 + e < rows) red_add_f32(p + (size_t)(c * 32 + e) * kD, __uint_as_float(v[c][e]));
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;\n" ::: "memory");
    // ------------------------------------------------------------ P / dS
    const int quad = warp & 3;
    const int r = quad * 32 + lane;                 // key row inside the tile (TMEM lane)
    const int tid = threadIdx.x - 256;              // 0..511
    const int g = tid >> 7;                         // which 16 queries of each half
    const int kv_pos = j * kTile + r;
    const uint32_t lane_base = tbase + ((uint32_t)(quad * 32) << 16);
    bool ok = true;
    // Every compute warp meets the named barrier below once per tile, also
    // after one of its bounded waits failed (it then skips the tile's work):
    // a warp leaving the loop early would leave the others waiting at it.
    for (int t = 0; t < n_it; ++t) {
      const int i = i0 + t;
      const int buf = t & 1;
      if (tid < kTile) {
        const int q = i * kTile + tid;
        sm->lse2[buf][tid] = q < S_q ? LSE[(size_t)bh * S_q + q] * 1.4426950408889634f : INFINITY;
        sm->delta[buf][tid] = q < S_q ? Delta[(size_t)bh * S_q + q] : 0.f;
      }
      named_bar_sync(1, 512);
      if (!ok) continue;
      const int q_lo = q_off + i * kTile;
      const bool need_mask = (j * kTile + kTile - 1 > q_lo) || (i * kTile + kTile > S_q) || (j * kTile + kTile > S_kv);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        ok = mbar_wait(&sm->s_ready[h], t & 1, abort);
        if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
        tc_fence_after();
        const int qc0 = h * 64 + g * 16;            // this warp's 16 query columns
        uint32_t s[16], dp[16], pk[8], dsw[8];
        tmem_ld16(lane_base + kColS + qc0, s);
        tmem_ld16(lane_base + kColDP + qc0, dp);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; e += 4) {
          const float4 L4 = *reinterpret_cast<const float4*>(&sm->lse2[buf][qc0 + e]);
          const float4 D4 = *reinterpret_cast<const float4*>(&sm->delta[buf][qc0 + e]);
          const float Ls[4] = {L4.x, L4.y, L4.z, L4.w};
          const float Ds[4] = {D4.x, D4.y, D4.z, D4.w};
          float pr[4], dr[4];
          const float2 sc2 = make_float2(scale2, scale2);
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            // two lanes at a time: arg = s*scale2 - lse2, dS = P * (dP - Delta)
            const float2 arg = ffma2(make_float2(__uint_as_float(s[e + u]), __uint_as_float(s[e + u + 1])), sc2,
                                     make_float2(-Ls[u], -Ls[u + 1]));
            float2 p = make_float2(ex2(arg.x), ex2(arg.y));
            if (need_mask) {
              const int ql = qc0 + e + u;
              const int qpos = q_lo + ql;
              if (kv_pos > qpos || i * kTile + ql >= S_q || kv_pos >= S_kv) p.x = 0.f;
              if (kv_pos > qpos + 1 || i * kTile + ql + 1 >= S_q || kv_pos >= S_kv) p.y = 0.f;
            }
            const float2 dd = fadd2(make_float2(__uint_as_float(dp[e + u]), __uint_as_float(dp[e + u + 1])),
                                    make_float2(-Ds[u], -Ds[u + 1]));
            const float2 ds = fmul2(p, dd);
            pr[u] = p.x; pr[u + 1] = p.y;
            dr[u] = ds.x; dr[u + 1] = ds.y;
          }
          pk[e / 2] = pack_bf16(pr[0], pr[1]);
          pk[e / 2 + 1] = pack_bf16(pr[2], pr[3]);
          dsw[e / 2] = pack_bf16(dr[0], dr[1]);
          dsw[e / 2 + 1] = pack_bf16(dr[2], dr[3]);
        }
#pragma unroll
        for (int v = 0; v < 2; ++v)
          st_sw128(sdS, r, qc0 / 8 + v, make_uint4(dsw[4 * v], dsw[4 * v + 1], dsw[4 * v + 2], dsw[4 * v + 3]));
        // P^T and dS^T as bf16 pairs into this warp's own 16 S^T columns (no
        // other warp reads them), where the dV / dK MMAs take them as A
        tmem_st8(lane_base + kColS + qc0, pk);
        tmem_st8(lane_base + kColS + qc0 + 8, dsw);
        tmem_st_wait();
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&sm->p_ready[h]);
      }
    }
    // epilogue: dV and dK rows of this key tile, once every MMA has completed
    if (!__any_sync(0xffffffffu, !ok)) {
      ok = n_it > 0 ? mbar_wait(&sm->mma_done, 0, abort) : true;
    }
    if (!__any_sync(0xffffffffu, !ok)) {
      tc_fence_after();
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = which == 0 ? kColDV : kColDK;
        const float mul = which == 0 ? 1.0f : scale;
        __nv_bfloat16* row = (which == 0 ? dV : dK) + ((size_t)bh * S_kv + kv_pos) * kD;
        {
          const int c = g;                          // this warp's 32 columns of dV / dK
          uint32_t v[32];
          if (n_it > 0) {
            tmem_ld32(lane_base + col + c * 32, v);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = 0u;
          }
          if (kv_pos < S_kv) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 w;
              w.x = pack_bf16(__uint_as_float(v[v4 * 8 + 0]) * mul, __uint_as_float(v[v4 * 8 + 1]) * mul);
              w.y = pack_bf16(__uint_as_float(v[v4 * 8 + 2]) * mul, __uint_as_float(v[v4 * 8 + 3]) * mul);
              w.z = pack_bf16(__uint_as_float(v[v4 * 8 + 4]) * mul, __uint_as_float(v[v4 * 8 + 5]) * mul);
              w.w = pack_bf16(__uint_as_float(v[v4 * 8 + 6]) * mul, __uint_as_float(v[v4 * 8 + 7]) * mul);
              *reinterpret_cast<uint4*>(row + c * 32 + v4 * 8) = w;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
  if (threadIdx.x == 0 && sm->abort) atomicExch(&g_attn_bwd_status, 1);
}

// Delta = rowsum(dO * O) in fp32; zero dQacc.  One warp per query row.
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ O, const __nv_bfloat16* __restrict__ dO,
                                     float* __restrict__ Delta, float* __restrict__ dQacc, long long rows) {
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const size_t off = (size_t)w * 128 + lane * 4;
  const uint2 a = *reinterpret_cast<const uint2*>(O + off);
  const uint2 b = *reinterpret_cast<const uint2*>(dO + off);
  const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
  float2 a0 = __bfloat1622float2(ha[0]), a1 = __bfloat1622float2(ha[1]);
  float2 b0 = __bfloat1622float2(hb[0]), b1 = __bfloat1622float2(hb[1]);
  float s = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  if (lane == 0) Delta[w] = s;
  *reinterpret_cast<float4*>(dQacc + off) = make_float4(0.f, 0.f, 0.f, 0.f);
}

__global__ void attn_bwd_post_kernel(const float* __restrict__ dQacc, __nv_bfloat16* __restrict__ dQ, float scale,
                                     long long n8) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(dQacc)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(dQacc)[2 * i + 1];
    uint4 w;
    w.x = pack_bf16(a.x * scale, a.y * scale);
    w.y = pack_bf16(a.z * scale, a.w * scale);
    w.z = pack_bf16(b.x * scale, b.y * scale);
    w.w = pack_bf16(b.z * scale, b.w * scale);
    reinterpret_cast<uint4*>(dQ)[i] = w;
  }
}

int attn_bwd_status(int reset) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, g_attn_bwd_status, sizeof(int));
  if (reset) { int z = 0; cudaMemcpyToSymbol(g_attn_bwd_status, &z, sizeof(int)); }
  return h;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t attn_bwd_workspace_size(int B, int H, int S_q, int S_kv, int D) {
  (void)S_kv;
  const size_t rows = (size_t)B * H * S_q;
  return align256(rows * D * sizeof(float)) + align256(rows * sizeof(float));
}

int attn_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse, const void* dO, int B,
             int H, int S_q, int S_kv, int q_off, int D, float scale, void* dq, void* dk, void* dv, void* ws,
             size_t ws_bytes, cudaStream_t st) {
  (void)ws_bytes;
  const size_t rows = (size_t)B * H * S_q;
  float* dQacc = reinterpret_cast<float*>(ws);
  float* Delta = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + align256(rows * D * sizeof(float)));
  CUtensorMap mq, mk, mv, mdo;
  int rc;
  if ((rc = make_tmap_rows(&mq, q, S_q, B * H, 64))) return rc;
  if ((rc = make_tmap_rows(&mk, k, S_kv, B * H, 128))) return rc;
  if ((rc = make_tmap_rows(&mv, v, S_kv, B * H, 128))) return rc;
  if ((rc = make_tmap_rows(&mdo, dO, S_q, B * H, 64))) return rc;
  {
    const long long threads = (long long)rows * 32;
    attn_bwd_prep_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)dO, Delta, dQacc, (long long)rows);
    if ((rc = check_launch("attn_bwd_prep_kernel"))) return rc;
  }
  const size_t smem = (3 + 2 * bwd::kStages) * bwd::kTileBytes + sizeof(BwdSmem);
  cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(B * H, (S_kv + bwd::kTile - 1) / bwd::kTile);
  attn_bwd_kernel<<<grid, bwd::kThreads, smem, st>>>(mq, mk, mv, mdo, lse, Delta, dQacc, (__nv_bfloat16*)dk,
                                                    (__nv_bfloat16*)dv, S_q, S_kv, q_off,
                                                    scale * 1.4426950408889634f, scale);
  if ((rc = check_launch("attn_bwd_kernel"))) return rc;
  const long long n8 = (long long)rows * D / 8;
  attn_bwd_post_kernel<<<148 * 8, 256, 0, st>>>(dQacc, (__nv_bfloat16*)dq, scale, n8);
  return check_launch("attn_bwd_post_kernel");
}

}  // namespace lh

namespace lh {

// ---------------------------------------------------------------------------
// Allocation-free variant of the attention backward.
//
// Some callers cannot allocate device memory at the point where they run the
// backward: a host runtime that hands the library only the tensors of the
// step (a JNI / cgo / C++ caller without access to PyTorch's caching
// allocator, for which cudaMalloc would also synchronise the device in the
// middle of a step), or a process whose memory pool is reserved up front and
// forbids new device allocations.  lh_attn_bwd_noalloc serves them: its
// workspace (the fp32 dQ accumulator and the per-row Delta) lives in the
// file-scope array below, which the CUDA runtime creates when the library is
// loaded on a device and keeps until the process exits.
//
// Limit: B*H*S_q <= kNoAllocMaxRows rows (8.4 MB per device).  Every call
// shares the array and it keeps the previous call's contents; the prep kernel
// rewrites all of it that a call reads (dQacc is zeroed, Delta recomputed).
// Calls that overlap on the GPU (different streams, or different threads
// without ordering) race on the array.
constexpr long long kNoAllocMaxRows = 16384;
constexpr size_t kNoAllocBytes = (size_t)kNoAllocMaxRows * 128 * sizeof(float) +
                                 (size_t)kNoAllocMaxRows * sizeof(float);
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch, looked up once per device (with that
// device current) on the first call made on it.
static void* noalloc_scratch_ptr(int* rc) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("attn_bwd_noalloc: no usable CUDA device");
    *rc = LH_ERR_LAUNCH;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("attn_bwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      *rc = LH_ERR_LAUNCH;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *rc = LH_OK;
  return ptrs[dev];
}

int attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse, const void* dO,
                     int B, int H, int S_q, int S_kv, int q_off, int D, float scale, void* dq, void* dk, void* dv,
                     cudaStream_t st) {
  if ((long long)B * H * S_q > kNoAllocMaxRows) {
    set_error("attn_bwd_noalloc: B*H*S_q = %lld rows exceeds the static workspace limit of %lld rows",
              (long long)B * H * S_q, kNoAllocMaxRows);
    return LH_ERR_SHAPE;
  }
  int rc = LH_OK;
  void* ws = noalloc_scratch_ptr(&rc);
  if (rc) return rc;
  // The workspace layout of attn_bwd: dQacc (rows x 128 fp32) then Delta, each 256-byte aligned.
  return attn_bwd(q, k, v, o, lse, dO, B, H, S_q, S_kv, q_off, D, scale, dq, dk, dv, ws, kNoAllocBytes, st);
}

}  // namespace lh
