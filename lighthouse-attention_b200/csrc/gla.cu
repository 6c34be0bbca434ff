// Simple gated linear attention, forward (the `gla` scorer's sequence mixer).
//
// The reference scorer DilatedLighthouseGLAScorer (src/lighthouse_selection.py:692-755)
// calls `chunk_simple_gla` of the external flash-linear-attention package
// (fla 0.5.1, fla/ops/simple_gla) twice, on dilated views of q/k/v with one
// scalar log-gate g per (token, head):
//     o_t = scale * sum_{s <= t} exp(G_t - G_s) (q_t . k_s) v_s,   G_t = sum_{i <= t} g_i
// i.e. the recurrence  S_t = exp(g_t) S_{t-1} + k_t v_t^T,  o_t = scale * q_t S_t
// with a zero initial state.  Layout (B, T, H, D), D = 128, bf16 in and out,
// fp32 gate (B, T, H).
//
// This kernel evaluates it chunk by chunk (C = 128 time steps) with the state held
// in fp32 registers for the whole sequence: one CTA per (batch, head, value
// slab of 64 columns, pass), eight warps, walking the chunks in order.  Per chunk
//     intra  A = (Q K^T) * scale * exp(G_t - G_s) [s <= t]        (C x C, fp32 -> bf16)
//     out    O = scale * exp(G_t) * (Q S_prev) + A V              (C x 64 slab)
//     state  S = exp(G_end) S_prev + (K * exp(G_end - G_s))^T V   (128 x 64 slab)
// with G chunk-local.  The products run on warp-level bf16 MMAs (m16n8k16,
// fp32 accumulate); the next chunk's Q/K/V stream into the other half of a
// double buffer with cp.async while the current one is computed, and one
// barrier per chunk orders the buffers.  The bf16-rounded operands (A, the
// decayed K, the state as the Q S operand) follow the
// precision of fla's chunked kernels.  Two (q, k, o) passes that share v and g
// (the scorer's q->k and k->q passes) run in one launch.
#include "lh_common.cuh"

namespace lh {
namespace gla {

#ifndef LH_GLA_CHUNK
#define LH_GLA_CHUNK 128
#endif
constexpr int C = LH_GLA_CHUNK; // chunk length (time steps): 64 or 128 (128 is faster: half the sequential steps)
constexpr int D = 128;         // head dim (key dim)
constexpr int VS = 64;         // value columns per CTA
constexpr int NT = 256;        // threads: eight warps
constexpr int NRB = C / 16;    // 16-row blocks of a chunk
constexpr int VH = 8 / NRB;    // warps sharing one row block (each takes VS / VH value columns)
constexpr int NO = VS / VH / 8; // 8-column output tiles per warp
static_assert(C == 64 || C == 128, "chunk of 64 or 128 steps");

struct Smem {
  __nv_bfloat16 q[2][C * D];   // rows of 256 B, 16-byte chunks XOR-swizzled by row
  __nv_bfloat16 k[2][C * D];
  __nv_bfloat16 v[2][C * VS];  // rows of 128 B
  __nv_bfloat16 st[2][D * VS]; // state S (key x value) as bf16, double-buffered
  float g2[2][C];              // chunk-local cumulative gate G, times log2(e)
  float kd[2][C];              // exp(G_end - G_s): decay of step s to the chunk end
};

__device__ __forceinline__ uint32_t sw256(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }
__device__ __forceinline__ uint32_t sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}

struct Pass {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  __nv_bfloat16* o;
};

// Issue the cp.async loads of chunk n (rows >= T are zero-filled).
__device__ __forceinline__ void load_chunk(Smem& sm, int buf, const Pass& ps, const __nv_bfloat16* v, int n, int T,
                                           long long row0, long long rstride, int vcol) {
  const uint32_t qs = (uint32_t)__cvta_generic_to_shared(sm.q[buf]);
  const uint32_t ks = (uint32_t)__cvta_generic_to_shared(sm.k[buf]);
  const uint32_t vs = (uint32_t)__cvta_generic_to_shared(sm.v[buf]);
  for (int i = threadIdx.x; i < C * 16; i += NT) {            // Q and K: 64 rows x 16 chunks
    const int r = i >> 4, c = i & 15, t = n * C + r;
    const bool ok = t < T;
    const long long off = ok ? (row0 + (long long)t * rstride) + c * 8 : 0;
    cp16(qs + sw256(r, c), ps.q + off, ok);
    cp16(ks + sw256(r, c), ps.k + off, ok);
  }
  for (int i = threadIdx.x; i < C * 8; i += NT) {             // V slab: 64 rows x 8 chunks
    const int r = i >> 3, c = i & 7, t = n * C + r;
    const bool ok = t < T;
    const long long off = ok ? (row0 + (long long)t * rstride) + vcol + c * 8 : 0;
    cp16(vs + sw128(r, c), v + off, ok);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Warp 0: chunk-local inclusive cumulative sum of g (lane holds steps lane + 32 i),
// times log2(e), and the decay of every step to the chunk end.
__device__ __forceinline__ void gate_scan(float* out, float* kd, float (&x)[C / 32], int lane) {
  constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int i = 0; i < C / 32; ++i) {
      const float y = __shfl_up_sync(0xffffffffu, x[i], o);
      if (lane >= o) x[i] += y;
    }
  }
#pragma unroll
  for (int i = 1; i < C / 32; ++i) x[i] += __shfl_sync(0xffffffffu, x[i - 1], 31);
  const float last = __shfl_sync(0xffffffffu, x[C / 32 - 1], 31) * kLog2e;
#pragma unroll
  for (int i = 0; i < C / 32; ++i) {
    out[lane + 32 * i] = x[i] * kLog2e;
    kd[lane + 32 * i] = exp2f(last - x[i] * kLog2e);
  }
}

__global__ void __launch_bounds__(NT, 1)
simple_gla_fwd_kernel(Pass p0, Pass p1, const __nv_bfloat16* __restrict__ v, const float* __restrict__ g, int T,
                      int H, int npass, float scale) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int slab = blockIdx.x, h = blockIdx.y;
  const int b = blockIdx.z / npass, pass = blockIdx.z - b * npass;
  const Pass ps = pass ? p1 : p0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;                     // mma fragment row / column pair
  // output rows 16rb.., slab columns vh * VS / VH..; rb mirrored for the upper four warps so
  // that the two warps of a scheduler (warp, warp + 4) hold one short and one long causal block
  const int half = warp >> 2;
  const int rb = half ? NRB - 1 - (warp & 3) : (warp & 3);
  const int vh = VH == 2 ? half : 0;
  const long long rstride = (long long)H * D;
  const long long row0 = ((long long)b * T * H + h) * D;     // element offset of (b, t = 0, h, 0)
  const int vcol = slab * VS;
  const int n_chunks = (T + C - 1) / C;
  const float* gh = g + (long long)b * T * H + h;            // g[b, t, h] = gh[t * H]

  // zero state operand for chunk 0 (it reads buffer 1)
  for (int i = threadIdx.x; i < D * VS / 2; i += NT) reinterpret_cast<uint32_t*>(sm.st[1])[i] = 0u;
  load_chunk(sm, 0, ps, v, 0, T, row0, rstride, vcol);
  float gn[C / 32];                                             // warp 0: gate of the next chunk
  if (warp == 0) {
#pragma unroll
    for (int i = 0; i < C / 32; ++i) gn[i] = lane + 32 * i < T ? gh[(long long)(lane + 32 * i) * H] : 0.f;
    gate_scan(sm.g2[0], sm.kd[0], gn, lane);
  }

  float sacc[8][4];                                            // state rows 16*warp.., 64 value columns
#pragma unroll
  for (int j = 0; j < 8; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;

  const uint32_t st_base[2] = {(uint32_t)__cvta_generic_to_shared(sm.st[0]),
                               (uint32_t)__cvta_generic_to_shared(sm.st[1])};

  for (int n = 0; n < n_chunks; ++n) {
    const int buf = n & 1;
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();                                           // chunk n, its gate scan and state n-1 visible
    if (n + 1 < n_chunks) {
      load_chunk(sm, buf ^ 1, ps, v, n + 1, T, row0, rstride, vcol);
      if (warp == 0) {
        const int t0 = (n + 1) * C;
#pragma unroll
        for (int i = 0; i < C / 32; ++i)
          gn[i] = t0 + lane + 32 * i < T ? gh[(long long)(t0 + lane + 32 * i) * H] : 0.f;
      }
    }
    const float* G = sm.g2[buf];
    const float gl = G[C - 1];
    const uint32_t qs = (uint32_t)__cvta_generic_to_shared(sm.q[buf]);
    const uint32_t ks = (uint32_t)__cvta_generic_to_shared(sm.k[buf]);
    const uint32_t vs = (uint32_t)__cvta_generic_to_shared(sm.v[buf]);

    // ---- intra scores A = Q K^T (rows 16rb.., causal key tiles only) and O_inter = Q S_prev
    float acc[2 * NRB][4], oacc[NO][4];
#pragma unroll
    for (int j = 0; j < 2 * NRB; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
    for (int j = 0; j < NO; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
    const uint32_t stp = buf ? st_base[0] : st_base[1];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      ldsm4(qs + sw256(16 * rb + (lane & 15), 2 * kk + (lane >> 4)), a);
#pragma unroll
      for (int np = 0; np < NRB; ++np) {
        if (np > rb) break;                                    // key tiles past the diagonal are masked
        uint32_t bb[4];
        ldsm4(ks + sw256(16 * np + (lane & 7) + ((lane >> 4) << 3), 2 * kk + ((lane >> 3) & 1)), bb);
        mma(acc[2 * np], a, bb[0], bb[1]);
        mma(acc[2 * np + 1], a, bb[2], bb[3]);
      }
#pragma unroll
      for (int np = 0; np < NO / 2; ++np) {
        uint32_t bb[4];
        ldsm4t(stp + sw128(16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3), NO * vh + 2 * np + (lane >> 4)), bb);
        mma(oacc[2 * np], a, bb[0], bb[1]);
        mma(oacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // scale the inter-chunk part by scale * exp(G_t); mask and decay the intra scores
    const int t_lo = 16 * rb + gq, t_hi = t_lo + 8;
    const float g_lo = G[t_lo], g_hi = G[t_hi];
    const float f_lo = scale * exp2f(g_lo), f_hi = scale * exp2f(g_hi);
#pragma unroll
    for (int j = 0; j < NO; ++j) {
      oacc[j][0] *= f_lo; oacc[j][1] *= f_lo; oacc[j][2] *= f_hi; oacc[j][3] *= f_hi;
    }
    uint32_t af[NRB][4];                                       // A as bf16 operand fragments, k-steps 0..rb
#pragma unroll
    for (int j = 0; j < 2 * NRB; ++j) {
      if ((j >> 1) > rb) break;
      const int s0 = 8 * j + 2 * tq, s1 = s0 + 1;
      const float gs0 = G[s0], gs1 = G[s1];
      const float x0 = s0 <= t_lo ? acc[j][0] * scale * exp2f(g_lo - gs0) : 0.f;
      const float x1 = s1 <= t_lo ? acc[j][1] * scale * exp2f(g_lo - gs1) : 0.f;
      const float x2 = s0 <= t_hi ? acc[j][2] * scale * exp2f(g_hi - gs0) : 0.f;
      const float x3 = s1 <= t_hi ? acc[j][3] * scale * exp2f(g_hi - gs1) : 0.f;
      af[j >> 1][(j & 1) * 2 + 0] = pack_bf16(x0, x1);
      af[j >> 1][(j & 1) * 2 + 1] = pack_bf16(x2, x3);
    }
    // ---- O += A V (k-steps over the causal key tiles)
#pragma unroll
    for (int kk = 0; kk < NRB; ++kk) {
      if (kk > rb) break;
      const uint32_t a[4] = {af[kk][0], af[kk][1], af[kk][2], af[kk][3]};
#pragma unroll
      for (int np = 0; np < NO / 2; ++np) {
        uint32_t bb[4];
        ldsm4t(vs + sw128(16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3), NO * vh + 2 * np + (lane >> 4)), bb);
        mma(oacc[2 * np], a, bb[0], bb[1]);
        mma(oacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // ---- store O (bf16): rows t_lo / t_hi, columns vcol + 8 (NO vh + j) + 2tq
    {
      const int ta = n * C + t_lo, tb = n * C + t_hi;
#pragma unroll
      for (int j = 0; j < NO; ++j) {
        const int col = vcol + 8 * (NO * vh + j) + 2 * tq;
        if (ta < T)
          *reinterpret_cast<uint32_t*>(ps.o + row0 + (long long)ta * rstride + col) = pack_bf16(oacc[j][0], oacc[j][1]);
        if (tb < T)
          *reinterpret_cast<uint32_t*>(ps.o + row0 + (long long)tb * rstride + col) = pack_bf16(oacc[j][2], oacc[j][3]);
      }
    }
    // ---- state S = exp(G_end) S + (K * exp(G_end - G_s))^T V; this warp: key rows 16*warp..
    const float fl = exp2f(gl);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sacc[j][0] *= fl; sacc[j][1] *= fl; sacc[j][2] *= fl; sacc[j][3] *= fl;
    }
#pragma unroll
    for (int kk = 0; kk < C / 16; ++kk) {
      uint32_t a[4];
      ldsm4t(ks + sw256(16 * kk + (lane & 7) + ((lane >> 4) << 3), 2 * warp + ((lane >> 3) & 1)), a);
      // fragment columns are steps s = 16kk + 2tq (+1) for a[0], a[1] and + 8 for a[2], a[3]
      const float2 d0 = *reinterpret_cast<const float2*>(&sm.kd[buf][16 * kk + 2 * tq]);
      const float2 d1 = *reinterpret_cast<const float2*>(&sm.kd[buf][16 * kk + 8 + 2 * tq]);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a[m]));
        const float2 d = m < 2 ? d0 : d1;
        a[m] = pack_bf16(x.x * d.x, x.y * d.y);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        ldsm4t(vs + sw128(16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3), 2 * np + (lane >> 4)), bb);
        mma(sacc[2 * np], a, bb[0], bb[1]);
        mma(sacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // bf16 copy of the state for the next chunk's Q S product
    {
      unsigned char* stb = reinterpret_cast<unsigned char*>(sm.st[buf]);
      const int r_lo = 16 * warp + gq, r_hi = r_lo + 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        *reinterpret_cast<uint32_t*>(stb + sw128(r_lo, j) + 4 * tq) = pack_bf16(sacc[j][0], sacc[j][1]);
        *reinterpret_cast<uint32_t*>(stb + sw128(r_hi, j) + 4 * tq) = pack_bf16(sacc[j][2], sacc[j][3]);
      }
    }
    if (warp == 0 && n + 1 < n_chunks) gate_scan(sm.g2[buf ^ 1], sm.kd[buf ^ 1], gn, lane);
  }
}

}  // namespace gla

int simple_gla_fwd(const void* q, const void* k, void* o, const void* q2, const void* k2, void* o2, const void* v,
                   const float* g, int B, int T, int H, float scale, cudaStream_t st) {
  using namespace gla;
  const int smem = (int)sizeof(Smem);
  cudaFuncSetAttribute(simple_gla_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int npass = q2 ? 2 : 1;
  const Pass p0{(const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (__nv_bfloat16*)o};
  const Pass p1 = q2 ? Pass{(const __nv_bfloat16*)q2, (const __nv_bfloat16*)k2, (__nv_bfloat16*)o2} : p0;
  simple_gla_fwd_kernel<<<dim3(D / VS, H, npass * B), NT, smem, st>>>(p0, p1, (const __nv_bfloat16*)v, g, T, H,
                                                                       npass, scale);
  return check_launch("simple_gla_fwd_kernel");
}

}  // namespace lh
