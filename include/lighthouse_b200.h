/*
 * lighthouse_b200 — C ABI of the B200 (sm_100a) Lighthouse selection-attention path.
 *
 * Every entry point takes device pointers, sizes and a cudaStream_t passed as
 * `void*` (NULL = legacy default stream), enqueues its kernels on that stream
 * and returns without synchronising.  No entry point allocates device memory:
 * outputs and workspaces are owned by the caller.  All tensors are dense and
 * row-major in the layout stated beside each argument.
 *
 * Return value: LH_OK (0) or an LH_ERR_* code; lh_last_error() then gives a
 * message for the calling thread.
 *
 * Layout names: B batch, S raw sequence length, H heads, D head dim (64 or
 * 128), L pyramid levels, p pooling factor (power of two), k top-k,
 * S_tot = sum_{l<L} S/p^l (pyramid length), S_pool = S_tot - S (levels >= 1),
 * S_sel = S/p^(L-1) + (L-1)*p*k (selected-sequence length).
 *
 * Reference files cited below are paths inside the reference project
 * (src/lighthouse_selection.py = SEL, src/lighthouse_selection_cuda.py = CU).
 */
#ifndef LIGHTHOUSE_B200_H
#define LIGHTHOUSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LH_OK = 0,
  LH_ERR_SHAPE = 1,   /* shape outside the supported / defined domain   */
  LH_ERR_ARG = 2,     /* null pointer, misaligned pointer, bad dtype      */
  LH_ERR_ARCH = 3,    /* device is not sm_100                             */
  LH_ERR_LAUNCH = 4,  /* CUDA launch / runtime error                      */
  LH_ERR_WORKSPACE = 5/* workspace too small                              */
};

enum { LH_DTYPE_BF16 = 0, LH_DTYPE_F32 = 1 };

/* Message for the last non-zero return on this thread ("" if none). */
const char* lh_last_error(void);

/* ABI version (major*100 + minor). */
int lh_abi_version(void);

/* 1 if an attention kernel on the current device left a bounded wait
 * (mbarrier spin limit) since the last reset, else 0.  Synchronises with the
 * device.  `reset` != 0 clears the flag. */
int lh_device_status(int reset);

/* Pyramid + norm scores.
 * Replaces DialatedLighthouseNormScorer.forward (SEL:589-616) and its CP twin
 * (SEL:955-982).
 *   xq, xk, xv        (B, S, H, D) dtype
 *   pooled_q/k/v      (B, H, S_pool, D) dtype: levels 1..L-1, level l = mean of
 *                     p^l consecutive raw tokens (fp32 accumulation)
 *   scores_qk/kq      (B, H, S_tot) fp32: level 0 = ||x||_2 over D rounded to
 *                     dtype, level l = max of the raw scores over p^l tokens
 * S must be a multiple of p^(L-1). */
int lh_pyramid_score_fwd(const void* xq, const void* xk, const void* xv, int dtype,
                         int B, int S, int H, int D, int L, int p,
                         void* pooled_q, void* pooled_k, void* pooled_v,
                         float* scores_qk, float* scores_kq, void* stream);

/* Hierarchical qk/kq chunked top-k selection in final position order.
 * Replaces LighthouseSelectionQkKqChunkedTopkNvrtc.forward (CU:359-429): the
 * NVRTC kernel (CU:114-330) plus its stable sort and gather (CU:425-427).
 *   scores_qk/kq  (B, H, S_tot) fp32
 *   indices       (B, H, S_sel) int32 out: pyramid indices in position order,
 *                 bit-identical to the reference's result
 *   inverse       (B, H, S_tot) int32 out, may be NULL: slot of each pyramid
 *                 entry in `indices`, -1 when not selected
 * Only the reference's defined domain is accepted: k % 128 == 0, p a power of
 * two with k/2 >= p, S/p^(L-1) divisible by T = k/128, NCC = S/p^(L-1)/T with
 * NCC >= 128 and NCC % 64 == 0 (LH_ERR_SHAPE otherwise). */
int lh_select_topk(const float* scores_qk, const float* scores_kq,
                   int B, int H, int S, int L, int p, int k,
                   int32_t* indices, int32_t* inverse, void* stream);

/* Inverse map from an index list (for callers holding only `indices`).
 *   indices (B, H, S_sel) int32 -> inverse (B, H, S_tot) int32 (-1 = absent) */
int lh_build_inverse(const int32_t* indices, int B, int H, int S_sel, int S_tot,
                     int32_t* inverse, void* stream);

/* Gather of the selected rows of Q, K and V from the pyramid.
 * Replaces the three torch.gather calls of SEL:800-813 (and SEL:1031-1042).
 *   x_raw    (B, S, H, D) dtype         level 0 of the pyramid (indices < S)
 *   x_pooled (B, H, S_pool, D) dtype    levels >= 1 (indices >= S)
 *   out      (B, H, S_sel, D) dtype
 * The three tensors are processed by one launch; any of the q/k/v triples
 * may be NULL to skip it. */
int lh_gather_selected(const void* q_raw, const void* k_raw, const void* v_raw,
                       const void* q_pooled, const void* k_pooled, const void* v_pooled,
                       int dtype, int B, int S, int H, int D, int S_pool,
                       const int32_t* indices, int S_sel,
                       void* q_sel, void* k_sel, void* v_sel, void* stream);

/* Causal attention forward over the selected sequence, softmax scale `scale`.
 * Replaces F.scaled_dot_product_attention(is_causal=True) at SEL:815 (via the
 * torchtitan wrapper, lighthouse-attention.patch:589,644), and, with q_off > 0,
 * one query chunk of the context-parallel ring (SEL:1044 under torch CP).
 * Query row r has causal position q_off + r, key row c has position c; row r
 * attends to keys c <= q_off + r, c < S_kv.  (q_off = 0, S_q = S_kv = S_sel is
 * plain causal attention.)
 *   q (B, H, S_q, D) bf16, k / v (B, H, S_kv, D) bf16, D == 128
 *   o (B, H, S_q, D) bf16; lse (B, H, S_q) fp32 natural-log logsumexp of the
 *   scaled scores. */
int lh_attn_fwd(const void* q, const void* k, const void* v, int B, int H, int S_q, int S_kv,
                int q_off, int D, float scale, void* o, float* lse, void* stream);

/* Log-sum-exp merge of two partial attentions of the same query rows over
 * disjoint key sets: the per-block results of the context-parallel attention
 * (SEL:1044 under torch's ring attention, whose merge is
 * torch/distributed/tensor/experimental/_context_parallel/_attention.py:71-77
 * and the ring loop at :380-470), here the local diagonal chunk and the
 * all-gathered earlier chunks.
 *   o1, o2 (rows, D) bf16; lse1, lse2 (rows) fp32 natural-log; D == 128
 *   o (rows, D) bf16, lse (rows) fp32 out (may alias o1 / lse1) */
int lh_attn_merge(const void* o1, const float* lse1, const void* o2, const float* lse2, long long rows,
                  int D, void* o, float* lse, void* stream);

/* Bytes of workspace lh_attn_bwd needs. */
size_t lh_attn_bwd_workspace_size(int B, int H, int S_q, int S_kv, int D);

/* Causal attention backward (dQ, dK, dV) for lh_attn_fwd (same geometry).
 *   do_ (B, H, S_q, D) bf16 upstream gradient of o
 *   dq (B, H, S_q, D), dk / dv (B, H, S_kv, D) bf16 out
 *   workspace  >= lh_attn_bwd_workspace_size bytes, 256-byte aligned */
int lh_attn_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse,
                const void* do_, int B, int H, int S_q, int S_kv, int q_off, int D, float scale,
                void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
                void* stream);

/* Allocation-free lh_attn_bwd, for callers that may not allocate device memory
 * during a step (a foreign-language host without PyTorch's caching allocator,
 * where cudaMalloc would also synchronise mid-step, or a process whose device
 * memory pool is fixed up front).  It has no counterpart in the reference.
 * Same arguments and results as lh_attn_bwd without the workspace: the
 * workspace is a static device array inside the library (8.4 MB per device,
 * held until the process exits).  Limit: B*H*S_q <= 16384 rows, else
 * LH_ERR_SHAPE.  The first call on a device looks up that array's address
 * (cudaGetSymbolAddress) with the device current; make that first call before
 * any stream capture.  All calls share the array: calls that overlap on the
 * GPU race with each other. */
int lh_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse,
                        const void* do_, int B, int H, int S_q, int S_kv, int q_off, int D, float scale,
                        void* dq, void* dk, void* dv, void* stream);

/* Fan-out of the selected outputs back to base positions (deterministic pull).
 * Replaces _ScatterToBaseAutograd.forward + _scatter_fanout_fwd_kernel
 * (SEL:408-459, 517-550): item s at pyramid level l with level-local position
 * j adds attn[s] to positions [j*p^l + p^l - 1, j*p^l + 2p^l - 1) of [0, N_total).
 *   attn    (B, H, S_sel, D) dtype
 *   inverse (B, H, S_tot) int32 (from lh_select_topk / lh_build_inverse),
 *           S_tot the pyramid length for N_shard
 *   out     (B, H, N_total, D) dtype (every element written) */
int lh_scatter_fwd(const void* attn, const int32_t* inverse, int dtype,
                   int B, int H, int S_sel, int D, int N_shard, int N_total, int L, int p,
                   void* out, void* stream);

/* Gather-sum adjoint of lh_scatter_fwd.
 * Replaces _ScatterToBaseAutograd.backward + _scatter_fanout_bwd_kernel
 * (SEL:462-514, 552-576).
 *   dout (B, H, N_total, D) dtype; indices (B, H, S_sel) int32;
 *   dattn (B, H, S_sel, D) dtype out. */
int lh_scatter_bwd(const void* dout, const int32_t* indices, int dtype,
                   int B, int H, int S_sel, int D, int N_shard, int N_total, int L, int p,
                   void* dattn, void* stream);

/* lh_scatter_fwd / lh_scatter_bwd with the base-position tensor in token-major
 * layout (B, N_total, H, D) instead of (B, H, N_total, D).  The reference's
 * call site transposes the layer output to (B, S, H*D) before the output
 * projection (lighthouse-attention.patch:737); written token-major, that
 * transpose is a view.  Needs D * element size of 256 or 512 bytes and
 * B*H divisible by the heads one warp covers (2 for bf16 D=128), else
 * LH_ERR_SHAPE. */
int lh_scatter_fwd_token_major(const void* attn, const int32_t* inverse, int dtype,
                               int B, int H, int S_sel, int D, int N_shard, int N_total,
                               int num_levels, int pooling_factor, void* out, void* stream);
int lh_scatter_bwd_token_major(const void* dout, const int32_t* indices, int dtype,
                               int B, int H, int S_sel, int D, int N_shard, int N_total,
                               int num_levels, int pooling_factor, void* dattn, void* stream);

/* Backward of gather + pyramid means: for each raw token t and head h,
 *   dx[b,t,h] = dsel[inv(t)] + sum_{l>=1} dsel[inv(off_l + t/p^l)] / p^l
 * (absent entries contribute 0).  Replaces the autograd of the three gathers
 * (SEL:800-813) and of the level means (SEL:604-606).
 *   dq_sel/dk_sel/dv_sel (B, H, S_sel, D) dtype; inverse (B, H, S_tot) int32;
 *   dxq/dxk/dxv (B, S, H, D) dtype out.  Any triple member may be NULL. */
int lh_unpool_bwd(const void* dq_sel, const void* dk_sel, const void* dv_sel,
                  const int32_t* inverse, int dtype, int B, int S, int H, int D, int L, int p,
                  int S_sel, void* dxq, void* dxk, void* dxv, void* stream);

/* Rotary position embedding of q and k (model harness; the reference applies
 * it in torchtitan's attention before the Lighthouse call, PATCH:700-737).
 *   xq, xk, oq, ok  (B, S, H, D) dtype (oq/ok may alias xq/xk)
 *   table           (S, D/2, 2) fp32 (cos, sin) per position and pair
 * Pairs (x[2i], x[2i+1]) rotate by the pair's angle; inverse != 0 rotates by
 * minus the angle (the backward). */
int lh_rope_apply(const void* xq, const void* xk, void* oq, void* ok, const float* table, int dtype,
                  int B, int S, int H, int D, int inverse, void* stream);

/* Simple gated linear attention forward, the sequence mixer of the `gla`
 * scorer: replaces fla.ops.simple_gla.chunk_simple_gla (fla 0.5.1) as called
 * by DilatedLighthouseGLAScorer.forward (src/lighthouse_selection.py:725-726)
 * with initial_state = None and output_final_state = False.
 *   q, k, v, o   (B, T, H, 128) bf16 (fla's head-last layout)
 *   g            (B, T, H) fp32 log-gate per step
 *   o_t = scale * sum_{s <= t} exp(G_t - G_s) (q_t . k_s) v_s,  G = cumsum(g)
 * A second (q2, k2, o2) triple sharing v and g runs in the same launch (the
 * scorer's q->k and k->q passes); pass NULL for all three to skip it. */
int lh_simple_gla_fwd(const void* q, const void* k, const void* v, const float* g, void* o, const void* q2,
                      const void* k2, void* o2, int dtype, int B, int T, int H, int D, float scale, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LIGHTHOUSE_B200_H */
