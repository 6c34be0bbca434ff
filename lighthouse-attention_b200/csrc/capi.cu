// extern "C" entry points of liblighthouse_b200.so (declared in
// include/lighthouse_b200.h).  Each validates its arguments, checks the device
// architecture once per device, and forwards to the kernel launcher.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "lh_common.cuh"

namespace lh {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return LH_ERR_LAUNCH;
  }
  return LH_OK;
}

// sm_100 check, cached per device.
static int check_arch() {
  static std::mutex mu;
  static int cached[64];  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { set_error("no CUDA device"); return LH_ERR_ARCH; }
  if (dev < 0 || dev >= 64) return LH_OK;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (cached[dev] == 0) {
      int major = 0, minor = 0;
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
      cached[dev] = (major == 10 && minor == 0) ? 1 : 2;
    }
    if (cached[dev] == 2) { set_error("lighthouse_b200 needs an sm_100 (B200) device"); return LH_ERR_ARCH; }
  }
  return LH_OK;
}

int pyramid_score_fwd(const void*, const void*, const void*, int, int, int, int, int, int, int, void*,
                      void*, void*, float*, float*, cudaStream_t);
int select_topk(const float*, const float*, int, int, int, int, int, int, int32_t*, int32_t*, cudaStream_t);
int gather_selected(const void*, const void*, const void*, const void*, const void*, const void*, int, int,
                    int, int, int, int, const int32_t*, int, void*, void*, void*, cudaStream_t);
int scatter_fwd(const void*, const int32_t*, int, int, int, int, int, int, int, int, int, void*, cudaStream_t);
int scatter_bwd(const void*, const int32_t*, int, int, int, int, int, int, int, int, int, void*, cudaStream_t);
int scatter_fwd_layout(const void*, const int32_t*, int, int, int, int, int, int, int, int, int, int, void*, cudaStream_t);
int scatter_bwd_layout(const void*, const int32_t*, int, int, int, int, int, int, int, int, int, int, void*, cudaStream_t);
int build_inverse(const int32_t*, int, int, int, int, int32_t*, cudaStream_t);
int unpool_bwd(const void*, const void*, const void*, const int32_t*, int, int, int, int, int, int, int, int,
               void*, void*, void*, cudaStream_t);
int attn_fwd(const void*, const void*, const void*, int, int, int, int, int, int, float, void*, float*,
             cudaStream_t);
size_t attn_bwd_workspace_size(int, int, int, int, int);
int attn_merge(const void*, const float*, const void*, const float*, long long, int, void*, float*, cudaStream_t);
int attn_status(int reset);
int rope_apply(const void*, const void*, void*, void*, const float*, int, int, int, int, int, int, cudaStream_t);
int simple_gla_fwd(const void*, const void*, void*, const void*, const void*, void*, const void*, const float*, int, int,
                   int, float, cudaStream_t);
int attn_bwd_noalloc(const void*, const void*, const void*, const void*, const float*, const void*, int, int, int,
                     int, int, int, float, void*, void*, void*, cudaStream_t);
int attn_bwd(const void*, const void*, const void*, const void*, const float*, const void*, int, int, int, int,
             int, int, float, void*, void*, void*, void*, size_t, cudaStream_t);

}  // namespace lh

using namespace lh;

#define LH_REQUIRE(cond, code, ...)         \
  do {                                      \
    if (!(cond)) {                          \
      set_error(__VA_ARGS__);               \
      return code;                          \
    }                                       \
  } while (0)

#define LH_ARCH()                 \
  do {                            \
    int _rc = check_arch();       \
    if (_rc) return _rc;          \
  } while (0)

static inline cudaStream_t S_(void* s) { return (cudaStream_t)s; }

extern "C" {

const char* lh_last_error(void) { return g_err; }

int lh_abi_version(void) { return 100; }

int lh_device_status(int reset) { return attn_status(reset); }

int lh_pyramid_score_fwd(const void* xq, const void* xk, const void* xv, int dtype, int B, int S, int H,
                         int D, int L, int p, void* pq, void* pk, void* pv, float* sqk, float* skq,
                         void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(xq && xk && xv && pq && pk && pv && sqk && skq, LH_ERR_ARG, "pyramid: null pointer");
  LH_REQUIRE(B > 0 && S > 0 && H > 0, LH_ERR_SHAPE, "pyramid: empty shape");
  LH_REQUIRE(p >= 2 && (p & (p - 1)) == 0, LH_ERR_SHAPE, "pyramid: pooling_factor must be a power of two >= 2");
  LH_REQUIRE(L >= 2 && L <= 6, LH_ERR_SHAPE, "pyramid: num_levels must be in [2, 6]");
  LH_REQUIRE(S % ipow(p, L - 1) == 0, LH_ERR_SHAPE, "pyramid: S must be a multiple of p^(L-1)");
  LH_ARCH();
  return pyramid_score_fwd(xq, xk, xv, dtype, B, S, H, D, L, p, pq, pk, pv, sqk, skq, S_(stream));
}

int lh_select_topk(const float* sqk, const float* skq, int B, int H, int S, int L, int p, int k,
                   int32_t* indices, int32_t* inverse, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(sqk && skq && indices, LH_ERR_ARG, "select: null pointer");
  LH_REQUIRE(B > 0 && H > 0 && S > 0, LH_ERR_SHAPE, "select: empty shape");
  LH_ARCH();
  return select_topk(sqk, skq, B, H, S, L, p, k, indices, inverse, S_(stream));
}

int lh_build_inverse(const int32_t* indices, int B, int H, int S_sel, int S_tot, int32_t* inverse,
                     void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(indices && inverse, LH_ERR_ARG, "build_inverse: null pointer");
  LH_ARCH();
  return build_inverse(indices, B, H, S_sel, S_tot, inverse, S_(stream));
}

int lh_gather_selected(const void* qr, const void* kr, const void* vr, const void* qp, const void* kp,
                       const void* vp, int dtype, int B, int S, int H, int D, int S_pool,
                       const int32_t* indices, int S_sel, void* qs, void* ks, void* vs, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(indices, LH_ERR_ARG, "gather: null indices");
  LH_REQUIRE(dtype == LH_DTYPE_BF16 || dtype == LH_DTYPE_F32, LH_ERR_ARG, "gather: bad dtype");
  LH_REQUIRE((!qs || (qr && qp)) && (!ks || (kr && kp)) && (!vs || (vr && vp)), LH_ERR_ARG,
             "gather: output given without its source tensors");
  LH_ARCH();
  return gather_selected(qr, kr, vr, qp, kp, vp, dtype, B, S, H, D, S_pool, indices, S_sel, qs, ks, vs, S_(stream));
}

int lh_attn_merge(const void* o1, const float* lse1, const void* o2, const float* lse2, long long rows, int D,
                  void* o, float* lse, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(o1 && lse1 && o2 && lse2 && o && lse, LH_ERR_ARG, "attn_merge: null pointer");
  LH_REQUIRE(D == 128, LH_ERR_SHAPE, "attn_merge: head dim must be 128, got %d", D);
  LH_REQUIRE(rows > 0, LH_ERR_SHAPE, "attn_merge: empty shape");
  LH_REQUIRE((((uintptr_t)o1 | (uintptr_t)o2 | (uintptr_t)o) & 7) == 0, LH_ERR_ARG, "attn_merge: rows must be 8-byte aligned");
  LH_ARCH();
  return attn_merge(o1, lse1, o2, lse2, rows, D, o, lse, S_(stream));
}

int lh_attn_fwd(const void* q, const void* k, const void* v, int B, int H, int S_q, int S_kv, int q_off, int D,
                float scale, void* o, float* lse, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(q && k && v && o && lse, LH_ERR_ARG, "attn_fwd: null pointer");
  LH_REQUIRE(D == 128, LH_ERR_SHAPE, "attn_fwd: head dim must be 128, got %d", D);
  LH_REQUIRE(B > 0 && H > 0 && S_q > 0 && S_kv > 0, LH_ERR_SHAPE, "attn_fwd: empty shape");
  LH_REQUIRE(q_off >= 0, LH_ERR_SHAPE, "attn_fwd: q_off must be >= 0");
  LH_ARCH();
  return attn_fwd(q, k, v, B, H, S_q, S_kv, q_off, D, scale, o, lse, S_(stream));
}

size_t lh_attn_bwd_workspace_size(int B, int H, int S_q, int S_kv, int D) {
  return attn_bwd_workspace_size(B, H, S_q, S_kv, D);
}

int lh_attn_bwd(const void* q, const void* k, const void* v, const void* o, const float* lse, const void* dO,
                int B, int H, int S_q, int S_kv, int q_off, int D, float scale, void* dq, void* dk, void* dv,
                void* ws, size_t ws_bytes, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(q && k && v && o && lse && dO && dq && dk && dv, LH_ERR_ARG, "attn_bwd: null pointer");
  LH_REQUIRE(D == 128, LH_ERR_SHAPE, "attn_bwd: head dim must be 128, got %d", D);
  LH_REQUIRE(B > 0 && H > 0 && S_q > 0 && S_kv > 0 && q_off >= 0, LH_ERR_SHAPE, "attn_bwd: bad shape");
  LH_REQUIRE(ws_bytes >= attn_bwd_workspace_size(B, H, S_q, S_kv, D), LH_ERR_WORKSPACE,
             "attn_bwd: workspace of %zu bytes is smaller than the %zu needed", ws_bytes,
             attn_bwd_workspace_size(B, H, S_q, S_kv, D));
  LH_REQUIRE(ws && ((uintptr_t)ws & 255) == 0, LH_ERR_ARG, "attn_bwd: workspace must be 256-byte aligned");
  LH_ARCH();
  return attn_bwd(q, k, v, o, lse, dO, B, H, S_q, S_kv, q_off, D, scale, dq, dk, dv, ws, ws_bytes, S_(stream));
}

int lh_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const float* lse,
                        const void* dO, int B, int H, int S_q, int S_kv, int q_off, int D, float scale, void* dq,
                        void* dk, void* dv, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(q && k && v && o && lse && dO && dq && dk && dv, LH_ERR_ARG, "attn_bwd_noalloc: null pointer");
  LH_REQUIRE(D == 128, LH_ERR_SHAPE, "attn_bwd_noalloc: head dim must be 128, got %d", D);
  LH_REQUIRE(B > 0 && H > 0 && S_q > 0 && S_kv > 0 && q_off >= 0, LH_ERR_SHAPE, "attn_bwd_noalloc: bad shape");
  LH_ARCH();
  return attn_bwd_noalloc(q, k, v, o, lse, dO, B, H, S_q, S_kv, q_off, D, scale, dq, dk, dv, S_(stream));
}

int lh_scatter_fwd(const void* attn, const int32_t* inverse, int dtype, int B, int H, int S_sel, int D,
                   int N_shard, int N_total, int L, int p, void* out, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(attn && inverse && out, LH_ERR_ARG, "scatter_fwd: null pointer");
  LH_REQUIRE(p >= 2 && (p & (p - 1)) == 0 && L >= 1 && L <= 7, LH_ERR_SHAPE, "scatter_fwd: bad L/p");
  LH_ARCH();
  return scatter_fwd(attn, inverse, dtype, B, H, S_sel, D, N_shard, N_total, L, p, out, S_(stream));
}

int lh_scatter_bwd(const void* dout, const int32_t* indices, int dtype, int B, int H, int S_sel, int D,
                   int N_shard, int N_total, int L, int p, void* dattn, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(dout && indices && dattn, LH_ERR_ARG, "scatter_bwd: null pointer");
  LH_REQUIRE(p >= 2 && (p & (p - 1)) == 0 && L >= 1 && L <= 7, LH_ERR_SHAPE, "scatter_bwd: bad L/p");
  LH_ARCH();
  return scatter_bwd(dout, indices, dtype, B, H, S_sel, D, N_shard, N_total, L, p, dattn, S_(stream));
}

int lh_scatter_fwd_token_major(const void* attn, const int32_t* inverse, int dtype, int B, int H, int S_sel, int D,
                               int N_shard, int N_total, int L, int p, void* out, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(attn && inverse && out, LH_ERR_ARG, "scatter_fwd: null pointer");
  LH_REQUIRE(p >= 2 && (p & (p - 1)) == 0 && L >= 1 && L <= 7, LH_ERR_SHAPE, "scatter_fwd: bad L/p");
  LH_ARCH();
  return scatter_fwd_layout(attn, inverse, dtype, B, H, S_sel, D, N_shard, N_total, L, p, 1, out, S_(stream));
}

int lh_scatter_bwd_token_major(const void* dout, const int32_t* indices, int dtype, int B, int H, int S_sel, int D,
                               int N_shard, int N_total, int L, int p, void* dattn, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(dout && indices && dattn, LH_ERR_ARG, "scatter_bwd: null pointer");
  LH_REQUIRE(p >= 2 && (p & (p - 1)) == 0 && L >= 1 && L <= 7, LH_ERR_SHAPE, "scatter_bwd: bad L/p");
  LH_ARCH();
  return scatter_bwd_layout(dout, indices, dtype, B, H, S_sel, D, N_shard, N_total, L, p, 1, dattn, S_(stream));
}

int lh_unpool_bwd(const void* dq, const void* dk, const void* dv, const int32_t* inverse, int dtype, int B,
                  int S, int H, int D, int L, int p, int S_sel, void* dxq, void* dxk, void* dxv, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(inverse, LH_ERR_ARG, "unpool_bwd: null inverse");
  LH_REQUIRE((!dxq || dq) && (!dxk || dk) && (!dxv || dv), LH_ERR_ARG, "unpool_bwd: output without input");
  LH_REQUIRE(p >= 2 && (p & (p - 1)) == 0 && L >= 1 && L <= 7, LH_ERR_SHAPE, "unpool_bwd: bad L/p");
  LH_ARCH();
  return unpool_bwd(dq, dk, dv, inverse, dtype, B, S, H, D, L, p, S_sel, dxq, dxk, dxv, S_(stream));
}

int lh_rope_apply(const void* xq, const void* xk, void* oq, void* ok, const float* table, int dtype, int B, int S,
                  int H, int D, int inverse, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(xq && xk && oq && ok && table, LH_ERR_ARG, "rope: null pointer");
  LH_REQUIRE(!(((uintptr_t)xq | (uintptr_t)xk | (uintptr_t)oq | (uintptr_t)ok | (uintptr_t)table) & 15), LH_ERR_ARG,
             "rope: pointers must be 16-byte aligned");
  LH_REQUIRE(dtype == LH_DTYPE_BF16 || dtype == LH_DTYPE_F32, LH_ERR_ARG, "rope: bad dtype");
  LH_REQUIRE(B > 0 && S > 0 && H > 0 && D > 0, LH_ERR_SHAPE, "rope: bad shape");
  LH_ARCH();
  return rope_apply(xq, xk, oq, ok, table, dtype, B, S, H, D, inverse, S_(stream));
}

int lh_simple_gla_fwd(const void* q, const void* k, const void* v, const float* g, void* o, const void* q2,
                      const void* k2, void* o2, int dtype, int B, int T, int H, int D, float scale, void* stream) {
  g_err[0] = 0;
  LH_REQUIRE(q && k && v && g && o, LH_ERR_ARG, "gla: null pointer");
  LH_REQUIRE((q2 == nullptr) == (k2 == nullptr) && (q2 == nullptr) == (o2 == nullptr), LH_ERR_ARG,
             "gla: q2, k2 and o2 must be given together");
  LH_REQUIRE(!(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o | (uintptr_t)q2 | (uintptr_t)k2 |
                (uintptr_t)o2) & 15) && !((uintptr_t)g & 3), LH_ERR_ARG, "gla: pointers must be 16-byte aligned");
  LH_REQUIRE(dtype == LH_DTYPE_BF16, LH_ERR_ARG, "gla: bf16 only");
  LH_REQUIRE(D == 128, LH_ERR_SHAPE, "gla: head_dim must be 128");
  LH_REQUIRE(B > 0 && T > 0 && H > 0 && B <= 32767 && H <= 65535, LH_ERR_SHAPE, "gla: bad shape");
  LH_ARCH();
  return simple_gla_fwd(q, k, o, q2, k2, o2, v, g, B, T, H, scale, S_(stream));
}

}  // extern "C"
