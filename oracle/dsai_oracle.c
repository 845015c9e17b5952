/*
 * dsai_oracle.c — CPU restatement of the reference DSA lightning indexer.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path and
 * the timed CPU baseline of bench.py; the product never links, loads or calls
 * it.  Parity status: see the header of oracle/oracle.py.
 *
 * It follows the reference's stated semantics:
 *   solution/python/kernel.cu:5-9 and solution/cuda/kernel.cu:4-21 (the math),
 *   solution/python/kernel.cu:29-40 (page layout: 8448 B = 64x128 e4m3 K, then
 *     64 fp32 scales at byte 8192; scale of slot s at 8192 + 4s),
 *   solution/python/kernel.cu:811-831 (epilogue order: ReLU, x weight, summed
 *     over heads, then x token scale; ReLU(x) = x > 0 ? x : 0, so NaN -> 0),
 *   solution/python/kernel.cu:855-859 (ordered keys, here the fp32 form),
 *   solution/python/kernel.cu:897-905, :1079-1097 (rows with seq_len <= 2048:
 *     physical ids of tokens 0..L-1 in token order, then -1),
 *   solution/python/kernel.cu:1021-1027 (physical id = bt[t/64]*64 + t%64).
 *
 * Arithmetic: e4m3 values are decoded exactly into doubles; each head score
 * S_h = sum_d q*k is exact in double (every product has <= 8 significant bits
 * and the partial sums stay within 53 bits), the head-weighted sum and the
 * scale are applied in double and the logit is rounded once to fp32.
 * Selection is exact: the K largest fp32 logits by ordered key, ties broken
 * by lower token index.
 *
 * Input conventions for malformed inputs (the reference leaves them
 * undefined): seq_len is clamped to [0, max_pages*64]; a block-table entry
 * outside [0, num_pages) reads as an all-zero page (K = 0, scale = 0).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define NH 64
#define HD 128
#define PS 64
#define TOPK 2048
#define PAGE_BYTES 8448
#define SCALE_OFF 8192

/* e4m3 (OCP FP8, "fn" variant): 1 sign, 4 exponent (bias 7), 3 mantissa
 * bits; no infinities; 0x7F / 0xFF are NaN; max finite 448. */
double dsai_oracle_e4m3(uint8_t x) {
  const int s = x >> 7, e = (x >> 3) & 0xF, m = x & 7;
  double v;
  if (e == 0xF && m == 7) return NAN;
  if (e == 0)
    v = ldexp((double)m, -9); /* subnormal: m/8 * 2^-6 */
  else
    v = ldexp(1.0 + m / 8.0, e - 7);
  return s ? -v : v;
}

static double g_tab[256];
static pthread_once_t g_tab_once = PTHREAD_ONCE_INIT;
static void init_tab(void) {
  for (int i = 0; i < 256; ++i) g_tab[i] = dsai_oracle_e4m3((uint8_t)i);
}

static int clamp_len(int L, int max_pages) {
  const int cap = max_pages * PS;
  return L < 0 ? 0 : (L > cap ? cap : L);
}

uint32_t dsai_oracle_key(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct {
  const uint8_t* q;
  const uint8_t* kc;
  const float* w;
  const int32_t* seq_lens;
  const int32_t* bt;
  int rows, max_pages, num_pages;
  float* logits;   /* [rows, max_pages*64] */
  float* mag;      /* optional [rows, max_pages*64]: scale * sum_h |ReLU(S_h) w_h| */
  int64_t n_items; /* work items: (row, 64-token page) */
  int64_t next;
  pthread_mutex_t mu;
} LogitJob;

static void score_page(LogitJob* J, int b, int pg) {
  const int ld = J->max_pages * PS;
  const int L = clamp_len(J->seq_lens[b], J->max_pages);
  const int t0 = pg * PS;
  if (t0 >= L) return;
  const int t1 = t0 + PS < L ? t0 + PS : L;
  double qd[NH][HD];
  const uint8_t* qb = J->q + (size_t)b * NH * HD;
  for (int h = 0; h < NH; ++h)
    for (int d = 0; d < HD; ++d) qd[h][d] = g_tab[qb[h * HD + d]];
  const int page = J->bt[(size_t)b * J->max_pages + pg];
  const int valid_page = page >= 0 && page < J->num_pages;
  for (int t = t0; t < t1; ++t) {
    const int slot = t - t0;
    double logit = 0.0, mag = 0.0;
    if (valid_page) {
      const uint8_t* kp = J->kc + (size_t)page * PAGE_BYTES;
      double kd[HD];
      for (int d = 0; d < HD; ++d) kd[d] = g_tab[kp[slot * HD + d]];
      float scale;
      memcpy(&scale, kp + SCALE_OFF + 4 * slot, 4);
      double acc = 0.0;
      for (int h = 0; h < NH; ++h) {
        /* four partial sums: every partial sum is exact, so the order is free */
        double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
        for (int d = 0; d < HD; d += 4) {
          s0 += qd[h][d] * kd[d];
          s1 += qd[h][d + 1] * kd[d + 1];
          s2 += qd[h][d + 2] * kd[d + 2];
          s3 += qd[h][d + 3] * kd[d + 3];
        }
        const double s = (s0 + s1) + (s2 + s3);
        const double r = s > 0.0 ? s : 0.0;
        const double wh = (double)J->w[(size_t)b * NH + h];
        acc += r * wh;
        mag += fabs(r * wh);
      }
      logit = acc * (double)scale;
      mag = mag * fabs((double)scale);
    }
    J->logits[(size_t)b * ld + t] = (float)logit;
    if (J->mag) J->mag[(size_t)b * ld + t] = (float)mag;
  }
}

static void* logit_worker(void* arg) {
  LogitJob* J = (LogitJob*)arg;
  for (;;) {
    pthread_mutex_lock(&J->mu);
    const int64_t i = J->next++;
    pthread_mutex_unlock(&J->mu);
    if (i >= J->n_items) break;
    score_page(J, (int)(i / J->max_pages), (int)(i % J->max_pages));
  }
  return NULL;
}

/* fp32 logits of every row and token t < L (all rows, short ones included);
 * entries at t >= L are set to -inf.  mag may be NULL.  Returns 0. */
int dsai_oracle_logits(const uint8_t* q, const uint8_t* k_cache, const float* weights,
                       const int32_t* seq_lens, const int32_t* block_table, int rows,
                       int max_pages, int num_pages, float* logits, float* mag, int nthreads) {
  pthread_once(&g_tab_once, init_tab);
  const size_t ld = (size_t)max_pages * PS;
  for (size_t i = 0; i < (size_t)rows * ld; ++i) {
    logits[i] = -INFINITY;
    if (mag) mag[i] = 0.0f;
  }
  LogitJob J;
  J.q = q;
  J.kc = k_cache;
  J.w = weights;
  J.seq_lens = seq_lens;
  J.bt = block_table;
  J.rows = rows;
  J.max_pages = max_pages;
  J.num_pages = num_pages;
  J.logits = logits;
  J.mag = mag;
  J.n_items = (int64_t)rows * max_pages;
  J.next = 0;
  pthread_mutex_init(&J.mu, NULL);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  for (int i = 1; i < nthreads; ++i) pthread_create(&th[i], NULL, logit_worker, &J);
  logit_worker(&J);
  for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
  pthread_mutex_destroy(&J.mu);
  return 0;
}

typedef struct {
  uint32_t key;
  int32_t idx;
} KeyIdx;

static int cmp_desc(const void* a, const void* b) {
  const KeyIdx* x = (const KeyIdx*)a;
  const KeyIdx* y = (const KeyIdx*)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

/* Sorts the first n entries (key desc, index asc) and keeps the top ones. */
static int top_entries(KeyIdx* e, int n) {
  qsort(e, (size_t)n, sizeof(KeyIdx), cmp_desc);
  return n < TOPK ? n : TOPK;
}

/* Top-2048 physical ids per row from fp32 logits [rows, max_pages*64].
 * Rows with L <= 2048: token order then -1.  Longer rows: descending logit
 * (ties by token index).  Returns 0, or -1 on allocation failure. */
int dsai_oracle_topk(const float* logits, const int32_t* seq_lens, const int32_t* block_table,
                     int rows, int max_pages, int32_t* out) {
  const size_t ld = (size_t)max_pages * PS;
  KeyIdx* e = (KeyIdx*)malloc(sizeof(KeyIdx) * (ld > 0 ? ld : 1));
  if (!e) return -1;
  for (int b = 0; b < rows; ++b) {
    const int L = clamp_len(seq_lens[b], max_pages);
    const int32_t* bt = block_table + (size_t)b * max_pages;
    int32_t* o = out + (size_t)b * TOPK;
    if (L <= TOPK) {
      for (int i = 0; i < TOPK; ++i) o[i] = i < L ? bt[i / PS] * PS + i % PS : -1;
      continue;
    }
    for (int t = 0; t < L; ++t) {
      e[t].key = dsai_oracle_key(logits[(size_t)b * ld + t]);
      e[t].idx = t;
    }
    const int n = top_entries(e, L);
    for (int i = 0; i < n; ++i) o[i] = bt[e[i].idx / PS] * PS + e[i].idx % PS;
  }
  free(e);
  return 0;
}

/* Per-row top-2048 (score, token + token_offset) pairs; rows with L <= 2048
 * give all tokens in token order then (-inf, -1).  Mirrors dsai_run_pairs. */
int dsai_oracle_pairs(const float* logits, const int32_t* seq_lens, int rows, int max_pages,
                      int32_t token_offset, float* out_scores, int32_t* out_tokens) {
  const size_t ld = (size_t)max_pages * PS;
  KeyIdx* e = (KeyIdx*)malloc(sizeof(KeyIdx) * (ld > 0 ? ld : 1));
  if (!e) return -1;
  for (int b = 0; b < rows; ++b) {
    const int L = clamp_len(seq_lens[b], max_pages);
    float* sc = out_scores + (size_t)b * TOPK;
    int32_t* tk = out_tokens + (size_t)b * TOPK;
    const float* row = logits + (size_t)b * ld;
    if (L <= TOPK) {
      for (int i = 0; i < TOPK; ++i) {
        sc[i] = i < L ? row[i] : -INFINITY;
        tk[i] = i < L ? i + token_offset : -1;
      }
      continue;
    }
    for (int t = 0; t < L; ++t) {
      e[t].key = dsai_oracle_key(row[t]);
      e[t].idx = t;
    }
    const int n = top_entries(e, L);
    for (int i = 0; i < n; ++i) {
      sc[i] = row[e[i].idx];
      tk[i] = e[i].idx + token_offset;
    }
  }
  free(e);
  return 0;
}

/* Merge of (score, token) candidates of one row into top-2048 physical ids,
 * as dsai_merge_pairs.  Token -1 is padding.  Ties by lower token. */
int dsai_oracle_merge(const float* scores, const int32_t* tokens, int n_cand,
                      const int32_t* bt_row, int max_pages, int32_t seq_len, int32_t* out) {
  const int L = clamp_len(seq_len, max_pages);
  if (L <= TOPK) {
    for (int i = 0; i < TOPK; ++i) out[i] = i < L ? bt_row[i / PS] * PS + i % PS : -1;
    return 0;
  }
  KeyIdx* e = (KeyIdx*)malloc(sizeof(KeyIdx) * (n_cand > 0 ? n_cand : 1));
  if (!e) return -1;
  int n = 0;
  for (int i = 0; i < n_cand; ++i)
    if (tokens[i] >= 0) {
      e[n].key = dsai_oracle_key(scores[i]);
      e[n].idx = tokens[i];
      ++n;
    }
  const int m = top_entries(e, n);
  for (int i = 0; i < TOPK; ++i) out[i] = i < m ? bt_row[e[i].idx / PS] * PS + e[i].idx % PS : -1;
  free(e);
  return 0;
}

/* ---------------------------------------------------------------- writer
 * CPU restatement of the index-K cache writer (the step that produces the
 * page layout above; the reference reads this format, solution/python/
 * kernel.cu:29-40, but has no writer).  Per token: amax = max |k| (at least
 * 1e-12), scale = amax / 448 in fp32, values clamp(k / scale, -448, 448)
 * rounded to e4m3 (round to nearest, ties to even).  The encoder follows the
 * e4m3 format definition: 1 sign bit, 4 exponent bits (bias 7), 3 mantissa
 * bits; exponent field 0 holds subnormals m * 2^-9; the largest finite value
 * is 448 (exponent 15, mantissa 6); exponent 15 with mantissa 7 is NaN. */
uint8_t dsai_oracle_e4m3_encode(float x) {
  const uint8_t sign = signbit(x) ? 0x80 : 0x00;
  double a = fabs((double)x);
  if (a > 448.0) a = 448.0;
  if (a == 0.0) return sign;
  unsigned code;
  if (a < ldexp(1.0, -6)) {          /* subnormal range: quantum 2^-9 */
    code = (unsigned)nearbyint(a * 512.0);  /* 8 carries into the smallest normal */
  } else {
    int e;
    (void)frexp(a, &e);              /* a in [2^(e-1), 2^e) */
    e -= 1;                          /* a in [2^e, 2^(e+1)) */
    unsigned q = (unsigned)nearbyint(ldexp(a, 3 - e));  /* in [8, 16] */
    if (q == 16) { q = 8; e += 1; }
    code = ((unsigned)(e + 7) << 3) | (q - 8);
  }
  if (code > 0x7E) code = 0x7E;      /* saturate at 448 */
  return (uint8_t)(sign | code);
}

int dsai_oracle_write_k(const float* k, int n, const int32_t* slot_ids, uint8_t* k_cache, int num_pages) {
  const long long num_slots = (long long)num_pages * PS;
  for (int i = 0; i < n; ++i) {
    const int32_t sid = slot_ids[i];
    if (sid < 0 || (long long)sid >= num_slots) continue;
    const float* v = k + (size_t)i * HD;
    float amax = 0.0f;
    for (int d = 0; d < HD; ++d) {
      const float m = fabsf(v[d]);
      if (m > amax) amax = m;
    }
    if (amax < 1e-12f) amax = 1e-12f;
    const float scale = amax / 448.0f;
    uint8_t* pg = k_cache + (size_t)(sid / PS) * PAGE_BYTES;
    const int slot = sid % PS;
    for (int d = 0; d < HD; ++d) {
      float x = v[d] / scale;
      if (x > 448.0f) x = 448.0f;
      if (x < -448.0f) x = -448.0f;
      pg[slot * HD + d] = dsai_oracle_e4m3_encode(x);
    }
    memcpy(pg + 8192 + 4 * slot, &scale, 4);
  }
  return 0;
}
