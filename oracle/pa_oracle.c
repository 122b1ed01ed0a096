/*
 * CPU oracle for paged-attention decode, in C with pthreads -- TEST
 * INFRASTRUCTURE ONLY (the checker and the timed CPU baseline; never linked
 * into or called by the shipped decode library).
 *
 * Restates the reference's fp32 oracle paged_attention_decode_reference
 * (src/reference.py:8-54) for contiguous inputs:
 *   for each sequence b with L = seq_lens[b] tokens:
 *     L == 0 -> output row is zero                     (src/reference.py:32-34)
 *     pages  = block_table[b, :ceil(L / page_size)]     (src/reference.py:36-42)
 *     K, V   = the first L token rows of those pages    (src/reference.py:43-44)
 *     query head h reads KV head h / (Hq / Hkv)         (src/reference.py:46-47)
 *     s = (q . k) * scale; s -= max(s); p = softmax(s); o = p @ V
 *                                                       (src/reference.py:49-52)
 * Work is split over (sequence, KV head) pairs across pthreads; all
 * arithmetic is fp32 like the reference. Inputs may be fp16 (raw IEEE
 * binary16 bits, converted exactly) or fp32.
 *
 * Pinned by tests/test_oracle_golden.py against outputs of the reference
 * itself (tests/golden/decode_golden.npz).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* Host threads the oracle uses by default: every online CPU. */
int pa_oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* Exact IEEE-754 binary16 -> binary32 conversion from the format's
 * definition (sign, 5-bit exponent bias 15, 10-bit fraction). */
static inline float half_bits_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t frac = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (frac == 0) {
      bits = sign;
    } else { /* subnormal: value = frac * 2^-24 */
      float f = (float)frac * (1.0f / 16777216.0f);
      memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (frac << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (frac << 13);
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

static inline void load_row(const void* base, int is_half, int64_t off, int64_t n, float* dst) {
  if (is_half) {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int64_t i = 0; i < n; ++i) dst[i] = half_bits_to_float(p[i]);
  } else {
    const float* p = (const float*)base + off;
    memcpy(dst, p, (size_t)n * sizeof(float));
  }
}

typedef struct {
  const void *q, *k, *v;
  int is_half;
  const int32_t *block_table, *seq_lens;
  float* out;
  int64_t batch, hq, hkv, d, num_pages, page_size, max_pages;
  float scale;
  int64_t next_pair; /* shared work cursor, taken with __atomic_fetch_add */
  int status;
} decode_job;

/* One worker: repeatedly claims a (sequence, KV head) pair and computes it. */
static void* decode_worker(void* arg) {
  decode_job* j = (decode_job*)arg;
  const int64_t g = j->hq / j->hkv, d = j->d, hq = j->hq, hkv = j->hkv;
  const int64_t pairs = j->batch * hkv;
  float* qrow = (float*)malloc(sizeof(float) * (size_t)(g * d));
  float* row = (float*)malloc(sizeof(float) * (size_t)d);
  float* acc = (float*)malloc(sizeof(float) * (size_t)(g * d));
  float* scores = NULL;
  int64_t scores_cap = 0;
  for (;;) {
    const int64_t pair = __atomic_fetch_add(&j->next_pair, 1, __ATOMIC_RELAXED);
    if (pair >= pairs) break;
    const int64_t b = pair / hkv, h = pair % hkv;
    const int64_t len = j->seq_lens[b];
    float* o = j->out + (b * hq + h * g) * d;
    if (len <= 0) {
      memset(o, 0, sizeof(float) * (size_t)(g * d));
      continue;
    }
    if (len > j->max_pages * j->page_size) {
      __atomic_store_n(&j->status, -3, __ATOMIC_RELAXED);
      continue;
    }
    if (scores_cap < g * len) {
      free(scores);
      scores_cap = g * len;
      scores = (float*)malloc(sizeof(float) * (size_t)scores_cap);
    }
    for (int64_t r = 0; r < g; ++r) load_row(j->q, j->is_half, (b * hq + h * g + r) * d, d, qrow + r * d);
    int bad = 0;
    /* scores = (q . k) * scale */
    for (int64_t t = 0; t < len; ++t) {
      const int64_t page = j->block_table[b * j->max_pages + t / j->page_size];
      if (page < 0 || page >= j->num_pages) { bad = 1; break; }
      load_row(j->k, j->is_half, ((page * j->page_size + t % j->page_size) * hkv + h) * d, d, row);
      for (int64_t r = 0; r < g; ++r) {
        float s = 0.f;
        const float* qq = qrow + r * d;
        for (int64_t i = 0; i < d; ++i) s += qq[i] * row[i];
        scores[r * len + t] = s * j->scale;
      }
    }
    if (bad) {
      __atomic_store_n(&j->status, -1, __ATOMIC_RELAXED);
      continue;
    }
    /* softmax with max subtraction */
    for (int64_t r = 0; r < g; ++r) {
      float* sr = scores + r * len;
      float mx = -INFINITY;
      for (int64_t t = 0; t < len; ++t) mx = sr[t] > mx ? sr[t] : mx;
      float sum = 0.f;
      for (int64_t t = 0; t < len; ++t) { sr[t] = expf(sr[t] - mx); sum += sr[t]; }
      const float inv = 1.0f / sum;
      for (int64_t t = 0; t < len; ++t) sr[t] *= inv;
    }
    /* o = p @ V */
    memset(acc, 0, sizeof(float) * (size_t)(g * d));
    for (int64_t t = 0; t < len; ++t) {
      const int64_t page = j->block_table[b * j->max_pages + t / j->page_size];
      load_row(j->v, j->is_half, ((page * j->page_size + t % j->page_size) * hkv + h) * d, d, row);
      for (int64_t r = 0; r < g; ++r) {
        const float p = scores[r * len + t];
        float* a = acc + r * d;
        for (int64_t i = 0; i < d; ++i) a[i] += p * row[i];
      }
    }
    memcpy(o, acc, sizeof(float) * (size_t)(g * d));
  }
  free(qrow);
  free(row);
  free(acc);
  free(scores);
  return NULL;
}

static int decode_impl(const void* q, const void* k, const void* v, int is_half,
                       const int32_t* block_table, const int32_t* seq_lens, float* out,
                       int64_t batch, int64_t hq, int64_t hkv, int64_t d, int64_t num_pages,
                       int64_t page_size, int64_t max_pages, float scale, int nthreads) {
  if (batch < 0 || hq <= 0 || hkv <= 0 || d <= 0 || page_size <= 0 || hq % hkv) return -2;
  decode_job job = {q, k, v, is_half, block_table, seq_lens, out, batch, hq, hkv, d,
                    num_pages, page_size, max_pages, scale, 0, 0};
  if (nthreads <= 0) nthreads = pa_oracle_max_threads();
  if (nthreads > 256) nthreads = 256;
  pthread_t tids[256];
  int started = 0;
  for (int i = 1; i < nthreads; ++i)
    if (pthread_create(&tids[started], NULL, decode_worker, &job) == 0) ++started;
  decode_worker(&job);
  for (int i = 0; i < started; ++i) pthread_join(tids[i], NULL);
  return job.status;
}

int pa_oracle_decode_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int32_t* block_table, const int32_t* seq_lens, float* out,
                         int64_t batch, int64_t hq, int64_t hkv, int64_t d, int64_t num_pages,
                         int64_t page_size, int64_t max_pages, float scale, int nthreads) {
  return decode_impl(q, k, v, 1, block_table, seq_lens, out, batch, hq, hkv, d, num_pages,
                     page_size, max_pages, scale, nthreads);
}

int pa_oracle_decode_f32(const float* q, const float* k, const float* v,
                         const int32_t* block_table, const int32_t* seq_lens, float* out,
                         int64_t batch, int64_t hq, int64_t hkv, int64_t d, int64_t num_pages,
                         int64_t page_size, int64_t max_pages, float scale, int nthreads) {
  return decode_impl(q, k, v, 0, block_table, seq_lens, out, batch, hq, hkv, d, num_pages,
                     page_size, max_pages, scale, nthreads);
}

