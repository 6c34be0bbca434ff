/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for Lighthouse selection.
 *
 * A plain-C restatement of the reference's hierarchical qk/kq chunked top-k
 * (src/lighthouse_selection_cuda.py, the kernel string at :114-330 and its
 * host wrapper at :359-429).  Only tests, the smoke check and bench.py's
 * CPU-baseline leg call it; the product library never links it.
 *
 * Restated pieces (reference file:line in src/lighthouse_selection_cuda.py):
 *   - float_to_ordered_uint / encode_key / encode_key_selected   :11-25
 *   - the 128-wide bitonic network, strict compares, desc=(i&k)==0 :41-110
 *     (the shuffle and shared-memory stages are the same comparator network,
 *      restated here as one loop over (k, j))
 *   - the per-tile level / batch loop                              :162-329
 *   - output sizes                                                 :346-357
 *   - the final stable sort by int32 key and gather of values      :425-427
 *
 * Two deliberate differences, both checked against the reference kernel on
 * the GPU by the GPU parity tests:
 *   - level_offset(level) is the exact integer sum_{j<level-1} N/p^j instead
 *     of the reference's fast-math float expression (:172-174);
 *   - 2^(1-level) is computed exactly (ldexpf).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TOPK 128
#define HALF 64

static uint32_t ordered_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (f >= 0.0f) ? (u ^ 0x80000000u) : ~u;
}

static uint32_t key_plain(int idx, int c_l) { return ordered_bits((float)(c_l * idx)); }

static uint32_t key_refined(int idx, int c_l, int level) {
  return ordered_bits((float)(c_l * (idx + 1)) - ldexpf(1.0f, 1 - level));
}

/* One bitonic network pass over 128 (score, index) pairs, descending. */
static void bitonic128_desc(float* s, int* ix) {
  for (int k = 2; k <= TOPK; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int lo = 0; lo < TOPK; ++lo) {
        int hi = lo ^ j;
        if (hi <= lo) continue;
        int desc = (lo & k) == 0;
        float a = s[lo], b = s[hi];
        int swap = desc ? (a < b) : (a > b);
        if (swap) {
          s[lo] = b; s[hi] = a;
          int t = ix[lo]; ix[lo] = ix[hi]; ix[hi] = t;
        }
      }
    }
  }
}

static long ipow(long b, int e) { long r = 1; while (e-- > 0) r *= b; return r; }

/* sum_{j=0}^{level-2} N / p^j : where level `level` starts in the pyramid */
static int level_offset(int N, int p, int level) {
  long off = 0;
  for (int j = 0; j < level - 1; ++j) off += N / ipow(p, j);
  return (int)off;
}

int lho_sel_len(int N, int L, int p, int k) {
  long total = 0;
  for (int level = L; level >= 1; --level) {
    if (level == L) total += N / ipow(p, level - 1);
    else total += (long)p * k;
  }
  return (int)total;
}

/* Runs one (b,h) tile.  keys/vals point at the (b,h) row of length S_sel. */
static void run_tile(const float* sq, const float* sk, int32_t* keys, int32_t* vals,
                     int S_sel, int tile, int N, int L, int p, int ncc, int chunk_len) {
  int parent[TOPK];
  float top_qk_s[HALF], top_kq_s[HALF];
  int top_qk_i[HALF], top_kq_i[HALF];
  float srt_s[TOPK];
  int srt_i[TOPK];
  int out_off = tile * chunk_len;
  int tile_start = tile * ncc;
  for (int i = 0; i < TOPK; ++i) parent[i] = -1;

#define EMIT(slot, key, val)                                   \
  do {                                                         \
    long _s = (slot);                                          \
    if (_s >= 0 && _s < S_sel) { keys[_s] = (int32_t)(key); vals[_s] = (val); } \
  } while (0)

  for (int level = L; level >= 1; --level) {
    int c_l = (int)ipow(p, level - 1);
    int K_end = N / c_l - 1;
    int lvl_off = level <= 1 ? 0 : level_offset(N, p, level);
    int ncand = (level == L) ? ncc : p * TOPK;
    int use_parents = level != L;
    int K_end_abs = K_end >= 0 ? K_end + lvl_off : -1;

#define CAND(col, out_idx)                                                  \
  do {                                                                      \
    int _c = (col);                                                         \
    int _k = -1;                                                            \
    if (_c < ncand) {                                                       \
      if (use_parents) {                                                    \
        int _pi = _c / p, _co = _c % p;                                     \
        int _pv = _pi < TOPK ? parent[_pi] : -1;                            \
        if (_pv >= 0) { _k = _pv * p + _co; if (_k > K_end || _k < 0) _k = -1; } \
      } else {                                                              \
        _k = tile_start + _c;                                               \
      }                                                                     \
    }                                                                       \
    (out_idx) = _k;                                                         \
  } while (0)
#define VALID(idx) ((idx) >= 0 && (idx) + lvl_off >= 0 && (idx) + lvl_off <= K_end_abs && K_end >= 0)

    if (level > 1) {
      for (int i = 0; i < HALF; ++i) {
        top_qk_s[i] = -1e6f; top_qk_i[i] = -1;
        top_kq_s[i] = -1e6f; top_kq_i[i] = -1;
      }
      int nb = (ncand + HALF - 1) / HALF;
      for (int b = 0; b < nb; ++b) {
        for (int i = 0; i < HALF; ++i) { srt_s[i] = top_qk_s[i]; srt_i[i] = top_qk_i[i]; }
        for (int i = 0; i < HALF; ++i) {
          int kidx;
          CAND(b * HALF + i, kidx);
          srt_s[HALF + i] = VALID(kidx) ? sq[kidx + lvl_off] : -1e6f;
          srt_i[HALF + i] = kidx;
        }
        bitonic128_desc(srt_s, srt_i);
        int rej[HALF];
        for (int i = 0; i < HALF; ++i) {
          top_qk_s[i] = srt_s[i]; top_qk_i[i] = srt_i[i];
          rej[i] = srt_i[HALF + i];
        }
        for (int i = 0; i < HALF; ++i) { srt_s[i] = top_kq_s[i]; srt_i[i] = top_kq_i[i]; }
        for (int i = 0; i < HALF; ++i) {
          srt_s[HALF + i] = VALID(rej[i]) ? sk[rej[i] + lvl_off] : -1e6f;
          srt_i[HALF + i] = rej[i];
        }
        bitonic128_desc(srt_s, srt_i);
        for (int i = 0; i < HALF; ++i) { top_kq_s[i] = srt_s[i]; top_kq_i[i] = srt_i[i]; }
        if (b >= 2) {
          for (int i = 0; i < HALF; ++i) {
            int d = srt_i[HALF + i];
            if (VALID(d)) EMIT(out_off + i, key_plain(d, c_l), d + lvl_off);
          }
          out_off += HALF;
        }
        if (b == nb - 1) {
          for (int i = 0; i < TOPK; ++i) {
            int t = i < HALF ? top_qk_i[i] : top_kq_i[i - HALF];
            if (t >= 0) EMIT(out_off + i, key_refined(t, c_l, level), t + lvl_off);
          }
          out_off += TOPK;
        }
      }
    } else {
      int nb = (ncand + TOPK - 1) / TOPK;
      for (int b = 0; b < nb; ++b) {
        for (int i = 0; i < TOPK; ++i) {
          int kidx;
          CAND(b * TOPK + i, kidx);
          if (VALID(kidx)) EMIT(out_off + i, key_plain(kidx, c_l), kidx + lvl_off);
        }
        int cnt = ncand - b * TOPK;
        out_off += cnt < TOPK ? cnt : TOPK;
      }
    }
    for (int i = 0; i < HALF; ++i) { parent[i] = top_qk_i[i]; parent[HALF + i] = top_kq_i[i]; }
#undef CAND
#undef VALID
  }
#undef EMIT
}

typedef struct { int32_t key; int32_t val; int32_t pos; } kv_t;

static int cmp_kv(const void* a, const void* b) {
  const kv_t* x = (const kv_t*)a;
  const kv_t* y = (const kv_t*)b;
  if (x->key != y->key) return x->key < y->key ? -1 : 1;
  return x->pos < y->pos ? -1 : (x->pos > y->pos);  /* stable */
}

/*
 * Selection over B*H rows.  scores_* are (B*H, S_tot) contiguous fp32.
 * keys_raw / vals_raw (optional, may be NULL) receive the unsorted
 * (key, value) slots as the reference kernel writes them; indices receives
 * the position-ordered result (B*H, S_sel).
 * Returns 0, or -1 when the shape is outside the reference's defined domain.
 */
int lho_select(const float* scores_qk, const float* scores_kq, int BH, int S_tot,
               int N, int L, int p, int k, int32_t* indices,
               int32_t* keys_raw, int32_t* vals_raw) {
  if (k % TOPK != 0 || (p & (p - 1)) != 0 || k / 2 < p || L < 1) return -1;
  int T = k / TOPK;
  long coarse = N;
  for (int i = 0; i < L - 1; ++i) coarse /= p;
  int ncc = (int)(coarse / T);
  if (ncc < TOPK) return -1;
  int S_sel = lho_sel_len(N, L, p, k);
  int chunk_len = lho_sel_len(N / T, L, p, TOPK);
  int32_t* keys = (int32_t*)malloc(sizeof(int32_t) * (size_t)S_sel);
  int32_t* vals = (int32_t*)malloc(sizeof(int32_t) * (size_t)S_sel);
  kv_t* kv = (kv_t*)malloc(sizeof(kv_t) * (size_t)S_sel);
  if (!keys || !vals || !kv) { free(keys); free(vals); free(kv); return -2; }
  for (int bh = 0; bh < BH; ++bh) {
    for (int i = 0; i < S_sel; ++i) { keys[i] = -1; vals[i] = -1; }
    const float* sq = scores_qk + (size_t)bh * S_tot;
    const float* sk = scores_kq + (size_t)bh * S_tot;
    for (int t = 0; t < T; ++t) run_tile(sq, sk, keys, vals, S_sel, t, N, L, p, ncc, chunk_len);
    if (keys_raw) memcpy(keys_raw + (size_t)bh * S_sel, keys, sizeof(int32_t) * S_sel);
    if (vals_raw) memcpy(vals_raw + (size_t)bh * S_sel, vals, sizeof(int32_t) * S_sel);
    for (int i = 0; i < S_sel; ++i) { kv[i].key = keys[i]; kv[i].val = vals[i]; kv[i].pos = i; }
    qsort(kv, (size_t)S_sel, sizeof(kv_t), cmp_kv);
    for (int i = 0; i < S_sel; ++i) indices[(size_t)bh * S_sel + i] = kv[i].val;
  }
  free(keys); free(vals); free(kv);
  return 0;
}
