/*
 * CPU oracle for the batched token sampler -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker / the timed CPU arm.  The
 * product path (mstar_rs_b200) never links or calls it.
 *
 * Parity status: UNPINNED.  The reference (npuichigo/mstar-rs) imports its
 * sampler from the external `mstar.utils.sampling` package, which is neither
 * vendored nor installed (python/mstar_rs/models/orpheus.py:78-83,
 * python/mstar_rs/models/qwen3_omni.py:405, :906-911) and ships no golden
 * vectors for sampling.  This file is a restatement of the sampler
 * *specification* built from the reference's call-site semantics:
 *   - greedy = temperature 0 / top_k 1      (orpheus.py:177-183, qwen3_omni.py:397-399)
 *   - repetition penalty over the request's generated-token set only
 *                                           (orpheus.py:187, :500)
 *   - per-request seed + per-slot RNG offset advanced in-graph
 *                                           (orpheus.py:353-359, qwen3_omni.py:485-496)
 *   - per-request params temperature/top_k/top_p/repetition_penalty
 *                                           (orpheus.py:177-185, qwen3_omni.py:1001-1009)
 * and the OpenAI / vLLM conventions for the knobs the reference forwards but
 * never sets itself (min_p, presence/frequency penalty, logit_bias, allowed
 * token bitmask; crates/mstar-server/src/adapters.rs:172-200).
 *
 * THE SPEC (every float op below is one IEEE-754 binary32 op, round to
 * nearest even, no fused multiply-add; f64 ops likewise in binary64):
 *
 *  1. v_i = logit_i as f32 (bf16 widened exactly).  NaN  -> excluded.
 *  2. logit_bias: for each bias entry (id, b) of the row, in list order,
 *     v_id = v_id + b.  Entries with id outside the row are ignored.
 *  3. penalties, only for tokens with occurrence count c_i > 0, where c_i is
 *     the number of times i appears among hist_ids[slot][0 .. min(len,H)),
 *     or (seen-bit mode) the token's bit in seen_bits[slot]:
 *        v = (v > 0) ? v / R : v * R          (repetition, R = rep_pen)
 *        v = v - (F * (float)c_i)             (frequency)
 *        v = v - P                            (presence)
 *  4. allowed bitmask: bit (i & 31) of word i >> 5 clear -> excluded.
 *  5. greedy iff !(T >= 1e-5): result = lowest id among non-excluded tokens
 *     whose v is maximal (ordered by okey, which equates -0 and +0).  If no
 *     such token exists or the max is -inf the row is EMPTY.
 *  6. otherwise x_i = v_i * fl(1/T); NaN -> excluded.
 *     m = max x over non-excluded tokens; no tokens or m == -inf -> EMPTY.
 *  7. order: (x descending, id ascending), i.e. ascending
 *        sortkey = ((u64)~okey(x) << 32) | id.
 *  8. e_i = 1 if x_i == m else E(x_i - m)      (E defined below)
 *     w_i = (u64) rint(e_i * 2^32)              (fixed-point weight)
 *  9. A = longest prefix of the order whose members all satisfy
 *        position < K            (top_k active: 0 < K)
 *        e_i >= min(Mp, 1)       (min_p active: Mp > 0)
 *        w_i > 0
 * 10. W_A = sum of w over A (exact u64).  top_p active iff P < 1:
 *        thr = (f64)P * (f64)W_A; keep the j-th member of A iff j == 0 or
 *        (f64)S_j < thr, S_j = sum of w of the members before it.
 *     Kept set K_set = that prefix (all of A when top_p is inactive).
 * 11. W_K = sum of w over K_set; u = uniforms[r] or Philox4x32-10 of
 *     (seed[slot], offset[slot]) (first output word, (x >> 8) * 2^-24);
 *        r = (u > 0) ? min((u64) floor((f64)u * (f64)W_K), W_K - 1) : 0;
 *     token = first member j of K_set with S_j + w_j > r.
 * 12. debug outputs: prob_j = (float)((f64)w_j / (f64)W_K) for members of
 *     K_set, else 0; kept_j = membership in K_set; x_j (v_j for greedy rows,
 *     -inf for excluded tokens except NaN inputs which stay NaN).
 * 13. EMPTY rows return token 0 (vocab_offset for shards) and set status bit 1.
 *
 * E(y), y <= 0  (exp written from the Taylor series of 2^f = e^{f ln 2}):
 *     t = y * L2E;  if t < -64 -> 0
 *     n = floor(t); f = t - n;  p = Horner(c8..c0, f) with c_k = fl((ln2)^k/k!)
 *     p = min(p, 2); return p * 2^n
 *   E is monotone non-decreasing and E(0) == 1, so A and K_set are prefixes.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_STATUS_EMPTY 1

static const float ORC_L2E = 0x1.715476p+0f;
static const float ORC_C[9] = {
    0x1.0p+0f,       0x1.62e43p-1f,   0x1.ebfbep-3f,   0x1.c6b08ep-5f,
    0x1.3b2ab6p-7f,  0x1.5d87fep-10f, 0x1.430912p-13f, 0x1.ffcbfcp-17f,
    0x1.62c022p-20f};

/* volatile stores keep gcc from contracting mul+add into an FMA. */
static float orc_mul(float a, float b) { volatile float r = a * b; return r; }
static float orc_add(float a, float b) { volatile float r = a + b; return r; }
static float orc_sub(float a, float b) { volatile float r = a - b; return r; }

static float orc_E(float y) {
  if (y == 0.0f) return 1.0f;
  float t = orc_mul(y, ORC_L2E);
  if (!(t >= -64.0f)) return 0.0f;
  float n = floorf(t);
  float f = orc_sub(t, n);
  float p = ORC_C[8];
  for (int k = 7; k >= 0; --k) p = orc_add(orc_mul(p, f), ORC_C[k]);
  if (p > 2.0f) p = 2.0f;
  return ldexpf(p, (int)n);
}

static uint32_t orc_fbits(float x) { uint32_t b; memcpy(&b, &x, 4); return b; }

static uint32_t orc_okey(float x) {
  uint32_t b = orc_fbits(x);
  if (b == 0x80000000u) b = 0;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

static uint64_t orc_weight(float x, float m, float *e_out) {
  float e = (x == m) ? 1.0f : orc_E(orc_sub(x, m));
  if (e_out) *e_out = e;
  float s = orc_mul(e, 4294967296.0f);
  return (uint64_t)rintf(s);
}

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
 * easy as 1, 2, 3", SC'11): 10 rounds of the 4x32 S-box with the published
 * multipliers and Weyl key increments. */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
  uint32_t k0 = key[0], k1 = key[1];
  for (int i = 0; i < 10; ++i) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* The sampler's draw: key = seed, counter = (offset lo, offset hi, 0, 0),
 * first output word. */
static uint32_t orc_philox_word0(uint64_t seed, uint64_t offset) {
  uint32_t ctr[4] = {(uint32_t)offset, (uint32_t)(offset >> 32), 0u, 0u};
  uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t out[4];
  orc_philox4x32_10(ctr, key, out);
  return out[0];
}

float orc_philox_uniform(uint64_t seed, uint64_t offset) {
  uint32_t w = orc_philox_word0(seed, offset);
  return (float)(w >> 8) * 0x1.0p-24f;
}

float orc_exp_spec(float y) { return orc_E(y); }

/* LSD radix sort of u64 keys, 16-bit digits; skips digits that are constant. */
static void orc_radix_sort_u64(uint64_t *a, uint64_t *tmp, int64_t n) {
  static const int DB = 16;
  size_t *cnt = (size_t *)malloc(sizeof(size_t) << DB);
  for (int pass = 0; pass < 4; ++pass) {
    int sh = pass * DB;
    memset(cnt, 0, sizeof(size_t) << DB);
    for (int64_t i = 0; i < n; ++i) cnt[(a[i] >> sh) & 0xFFFF]++;
    int constant = 0;
    for (size_t d = 0; d < (1u << DB); ++d)
      if (cnt[d] == (size_t)n) { constant = 1; break; }
    if (constant) continue;
    size_t acc = 0;
    for (size_t d = 0; d < (1u << DB); ++d) { size_t c = cnt[d]; cnt[d] = acc; acc += c; }
    for (int64_t i = 0; i < n; ++i) tmp[cnt[(a[i] >> sh) & 0xFFFF]++] = a[i];
    memcpy(a, tmp, (size_t)n * sizeof(uint64_t));
  }
  free(cnt);
}

typedef struct {
  const void *logits;      /* [B, ld] row-major, f32 (dtype 0) or bf16 (dtype 1) */
  int dtype;
  int64_t ld;
  int32_t B, V;
  int64_t vocab_offset;    /* global id of column 0 */
  const int32_t *slot_idx; /* [B] or NULL (row r uses slot r); slot < 0 skips the row */
  const float *temperature, *top_p, *min_p, *rep_pen, *pres_pen, *freq_pen; /* [slots] */
  const int32_t *top_k;                                                    /* [slots] */
  const int32_t *hist_ids; const int32_t *hist_len; int32_t H;             /* global ids */
  const uint32_t *seen_bits; int64_t seen_words;                           /* global ids */
  const int32_t *bias_ids; const float *bias_vals; int32_t NB;             /* global ids */
  const uint32_t *allowed_bits; int64_t allowed_words;                     /* global ids */
  const float *uniforms;                                                   /* [B] or NULL */
  const uint64_t *seed, *offset;                                           /* [slots] */
  int64_t *out_ids;      /* [B] */
  int32_t *out_status;   /* [B] or NULL */
  float *out_probs;      /* [B, V] or NULL */
  uint8_t *out_kept;     /* [B, V] or NULL */
  float *out_x;          /* [B, V] or NULL */
} orc_args_t;

static float orc_load(const orc_args_t *a, int64_t r, int64_t i) {
  if (a->dtype == 0) return ((const float *)a->logits)[r * a->ld + i];
  uint16_t h = ((const uint16_t *)a->logits)[r * a->ld + i];
  uint32_t b = (uint32_t)h << 16;
  float f; memcpy(&f, &b, 4); return f;
}

static void orc_row(const orc_args_t *a, int64_t r) {
  const int64_t V = a->V, off = a->vocab_offset;
  int32_t slot = a->slot_idx ? a->slot_idx[r] : (int32_t)r;
  if (a->out_probs) memset(a->out_probs + r * V, 0, (size_t)V * sizeof(float));
  if (a->out_kept) memset(a->out_kept + r * V, 0, (size_t)V);
  if (slot < 0) {
    a->out_ids[r] = off;
    if (a->out_status) a->out_status[r] = 0;
    if (a->out_x) for (int64_t i = 0; i < V; ++i) a->out_x[r * V + i] = -INFINITY;
    return;
  }
  float *v = (float *)malloc((size_t)V * sizeof(float));
  uint8_t *excl = (uint8_t *)calloc((size_t)V, 1);
  int32_t *cnt = (int32_t *)calloc((size_t)V, sizeof(int32_t));
  for (int64_t i = 0; i < V; ++i) {
    v[i] = orc_load(a, r, i);
    if (isnan(v[i])) excl[i] = 1;
  }
  /* 2. logit bias in list order */
  if (a->bias_ids) {
    for (int32_t j = 0; j < a->NB; ++j) {
      int64_t id = (int64_t)a->bias_ids[(int64_t)slot * a->NB + j] - off;
      if (id < 0 || id >= V) continue;
      v[id] = orc_add(v[id], a->bias_vals[(int64_t)slot * a->NB + j]);
    }
  }
  /* 3. penalties */
  if (a->hist_ids) {
    int32_t len = a->hist_len[slot];
    int32_t n = len < a->H ? len : a->H;
    for (int32_t j = 0; j < n; ++j) {
      int64_t id = (int64_t)a->hist_ids[(int64_t)slot * a->H + j] - off;
      if (id >= 0 && id < V) cnt[id]++;
    }
  } else if (a->seen_bits) {
    for (int64_t i = 0; i < V; ++i) {
      int64_t g = i + off;
      cnt[i] = (a->seen_bits[(int64_t)slot * a->seen_words + (g >> 5)] >> (g & 31)) & 1u;
    }
  }
  const float R = a->rep_pen ? a->rep_pen[slot] : 1.0f;
  const float F = a->freq_pen ? a->freq_pen[slot] : 0.0f;
  const float P = a->pres_pen ? a->pres_pen[slot] : 0.0f;
  for (int64_t i = 0; i < V; ++i) {
    if (cnt[i] <= 0) continue;
    float x = v[i];
    x = (x > 0.0f) ? (float)(x / R) : orc_mul(x, R);
    x = orc_sub(x, orc_mul(F, (float)cnt[i]));
    x = orc_sub(x, P);
    v[i] = x;
  }
  for (int64_t i = 0; i < V; ++i)
    if (isnan(v[i])) excl[i] = 1;
  /* 4. allowed bitmask */
  if (a->allowed_bits) {
    for (int64_t i = 0; i < V; ++i) {
      int64_t g = i + off;
      if (!((a->allowed_bits[(int64_t)slot * a->allowed_words + (g >> 5)] >> (g & 31)) & 1u))
        excl[i] = 1;
    }
  }
  const float T = a->temperature ? a->temperature[slot] : 1.0f;
  int greedy = !(T >= 1e-5f);
  int64_t tok = -1;
  int status = 0;
  if (greedy) {
    uint32_t best = 0; int have = 0;
    for (int64_t i = 0; i < V; ++i) {
      if (excl[i]) continue;
      uint32_t k = orc_okey(v[i]);
      if (!have || k > best) { best = k; tok = i; have = 1; }
    }
    if (!have || v[tok] == -INFINITY) { tok = -1; }
    if (a->out_x)
      for (int64_t i = 0; i < V; ++i)
        a->out_x[r * V + i] = excl[i] ? (isnan(v[i]) ? v[i] : -INFINITY) : v[i];
    if (tok >= 0) {
      if (a->out_kept) a->out_kept[r * V + tok] = 1;
      if (a->out_probs) a->out_probs[r * V + tok] = 1.0f;
    }
  } else {
    const float invT = (float)(1.0f / T);
    float m = -INFINITY; int have = 0;
    for (int64_t i = 0; i < V; ++i) {
      if (excl[i]) continue;
      float x = orc_mul(v[i], invT);
      v[i] = x;
      if (isnan(x)) { excl[i] = 1; continue; }
      if (!have || x > m) m = x;
      have = 1;
    }
    if (a->out_x)
      for (int64_t i = 0; i < V; ++i)
        a->out_x[r * V + i] = excl[i] ? (isnan(v[i]) ? v[i] : -INFINITY) : v[i];
    if (have && m != -INFINITY) {
      /* candidates: w > 0 only (everything else can never be in A) */
      int64_t n = 0;
      uint64_t *keys = (uint64_t *)malloc((size_t)V * sizeof(uint64_t));
      for (int64_t i = 0; i < V; ++i) {
        if (excl[i]) continue;
        if (orc_weight(v[i], m, NULL) == 0) continue;
        keys[n++] = ((uint64_t)(~orc_okey(v[i])) << 32) | (uint64_t)i;
      }
      uint64_t *tmp = (uint64_t *)malloc((size_t)(n > 0 ? n : 1) * sizeof(uint64_t));
      orc_radix_sort_u64(keys, tmp, n);
      const int32_t K = a->top_k ? a->top_k[slot] : 0;
      float Mp = a->min_p ? a->min_p[slot] : 0.0f;
      const int minp_on = Mp > 0.0f;
      if (Mp > 1.0f) Mp = 1.0f;
      const float Pp = a->top_p ? a->top_p[slot] : 1.0f;
      int64_t nA = n;
      if (K > 0 && (int64_t)K < nA) nA = K;
      uint64_t *w = tmp; /* reuse */
      for (int64_t j = 0; j < nA; ++j) {
        int64_t id = (int64_t)(keys[j] & 0xFFFFFFFFu);
        float e;
        w[j] = orc_weight(v[id], m, &e);
        if (minp_on && !(e >= Mp)) { nA = j; break; }
      }
      uint64_t WA = 0;
      for (int64_t j = 0; j < nA; ++j) WA += w[j];
      int64_t nK = nA;
      if (Pp < 1.0f) {
        double thr = (double)Pp * (double)WA;
        uint64_t S = 0; int64_t j = 0;
        for (; j < nA; ++j) {
          if (j > 0 && !((double)S < thr)) break;
          S += w[j];
        }
        nK = j;
      }
      uint64_t WK = 0;
      for (int64_t j = 0; j < nK; ++j) WK += w[j];
      float u;
      if (a->uniforms) u = a->uniforms[r];
      else u = orc_philox_uniform(a->seed[slot], a->offset[slot]);
      uint64_t rr = 0;
      if (u > 0.0f) {
        double t = floor((double)u * (double)WK);
        rr = (t >= (double)WK) ? WK - 1 : (uint64_t)t;
      }
      uint64_t S = 0;
      for (int64_t j = 0; j < nK; ++j) {
        if (S + w[j] > rr) { tok = (int64_t)(keys[j] & 0xFFFFFFFFu); break; }
        S += w[j];
      }
      for (int64_t j = 0; j < nK; ++j) {
        int64_t id = (int64_t)(keys[j] & 0xFFFFFFFFu);
        if (a->out_kept) a->out_kept[r * V + id] = 1;
        if (a->out_probs) a->out_probs[r * V + id] = (float)((double)w[j] / (double)WK);
      }
      free(keys); free(tmp);
    }
  }
  if (tok < 0) { status |= ORC_STATUS_EMPTY; tok = 0; }
  a->out_ids[r] = tok + off;
  if (a->out_status) a->out_status[r] = status;
  free(v); free(excl); free(cnt);
}

int orc_sample(const orc_args_t *a, int nthreads) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
  for (int64_t r = 0; r < a->B; ++r) orc_row(a, r);
  return 0;
}

int orc_args_size(void) { return (int)sizeof(orc_args_t); }
