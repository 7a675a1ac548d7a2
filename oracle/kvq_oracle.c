/*
 * CPU oracle for the 4-bit KV-cache hot path, plain C (test infrastructure).
 *
 * This is the checker and the CPU baseline, never the product: only the tests,
 * the smoke check and the benchmark's CPU-baseline leg load it.
 *
 * It restates the reference torch path of sztlink/krea-realtime-bench:
 *   kvqo_quantize    QuantKVTensor._quantize   quant_kv.py:142-159
 *   kvqo_dequantize  QuantKVTensor._dequantize quant_kv.py:161-176
 * with the same arithmetic contract as oracle/kvq_oracle.py: fp32 amax over bf16
 * values, IEEE fp32 divides (amax / qmax and x / s with the unrounded scale),
 * round-half-to-even, bf16(scale) with round-to-nearest-even.
 *
 * Build with -O2 -ffp-contract=off and without -ffast-math: the divides and the
 * rounding must stay IEEE.
 *
 * kvqo_check_fast_codes() is an exhaustive proof helper: the code of an element
 * depends only on the pair (x, amax), both bf16, so every case can be enumerated.
 * It checks that the division-free formula the CUDA kernel uses gives the same
 * code as the reference formula for every finite pair with |x| <= amax.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (isnan(f)) return 0x7FC0;
  uint32_t bias = 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)((u + bias) >> 16);
}

/* NaN-propagating max, like torch.amax (quant_kv.py:151). */
static inline float nan_max(float m, float a) { return (a > m || isnan(a)) ? a : m; }

typedef struct {
  const uint16_t* x;
  int64_t x_row_stride; /* elements between consecutive tokens */
  uint8_t* codes;
  uint16_t* scales;
  int64_t t0, t1; /* token range */
  int H, D, G, bits;
  const int32_t* edges; /* 2*G ints: lo, hi */
} qjob_t;

static void quantize_rows(const qjob_t* j) {
  const int qmax = (1 << (j->bits - 1)) - 1;
  const int D = j->D, H = j->H, G = j->G;
  const int cw = j->bits == 4 ? D / 2 : D;
  float xf[1024];
  int16_t q[1024];
  for (int64_t t = j->t0; t < j->t1; ++t) {
    for (int h = 0; h < H; ++h) {
      const uint16_t* xr = j->x + t * j->x_row_stride + (int64_t)h * D;
      uint8_t* cr = j->codes + (t * H + h) * (int64_t)cw;
      uint16_t* sr = j->scales + (t * H + h) * (int64_t)G;
      for (int c = 0; c < D; ++c) xf[c] = bf16_to_f32(xr[c]);
      for (int g = 0; g < G; ++g) {
        int lo = j->edges[2 * g], hi = j->edges[2 * g + 1];
        float m = 0.0f;
        for (int c = lo; c < hi; ++c) m = nan_max(m, fabsf(xf[c]));
        float s = m / (float)qmax;
        if (!(s > 0.0f)) s = 1.0f;
        for (int c = lo; c < hi; ++c) {
          float r = nearbyintf(xf[c] / s);
          if (r > (float)qmax) r = (float)qmax;
          if (r < (float)-qmax) r = (float)-qmax;
          q[c] = (int16_t)r;
        }
        sr[g] = f32_to_bf16(s);
      }
      if (j->bits == 8) {
        for (int c = 0; c < D; ++c) cr[c] = (uint8_t)(q[c] + 128);
      } else {
        for (int i = 0; i < D / 2; ++i)
          cr[i] = (uint8_t)((q[2 * i] + 8) | ((q[2 * i + 1] + 8) << 4));
      }
    }
  }
}

typedef struct {
  const uint8_t* codes;
  const uint16_t* scales;
  uint16_t* out;
  int64_t t0, t1;
  int H, D, G, bits;
  const int32_t* edges;
} djob_t;

static void dequantize_rows(const djob_t* j) {
  const int D = j->D, H = j->H, G = j->G;
  const int cw = j->bits == 4 ? D / 2 : D;
  int16_t q[1024];
  for (int64_t t = j->t0; t < j->t1; ++t) {
    for (int h = 0; h < H; ++h) {
      const uint8_t* cr = j->codes + (t * H + h) * (int64_t)cw;
      const uint16_t* sr = j->scales + (t * H + h) * (int64_t)G;
      uint16_t* orow = j->out + (t * H + h) * (int64_t)D;
      if (j->bits == 8) {
        for (int c = 0; c < D; ++c) q[c] = (int16_t)cr[c] - 128;
      } else {
        for (int i = 0; i < D / 2; ++i) {
          q[2 * i] = (int16_t)(cr[i] & 0x0F) - 8;
          q[2 * i + 1] = (int16_t)((cr[i] >> 4) & 0x0F) - 8;
        }
      }
      for (int g = 0; g < G; ++g) {
        float s = bf16_to_f32(sr[g]);
        for (int c = j->edges[2 * g]; c < j->edges[2 * g + 1]; ++c)
          orow[c] = f32_to_bf16((float)q[c] * s);
      }
    }
  }
}

static void* q_thread(void* p) { quantize_rows((const qjob_t*)p); return NULL; }
static void* d_thread(void* p) { dequantize_rows((const djob_t*)p); return NULL; }

#define KVQO_MAX_THREADS 256

/* x: [L tokens][H][D] bf16 bits with x_row_stride elements between tokens.
 * codes: [L][H][D/2] (int4) or [L][H][D] (int8); scales: [L][H][G] bf16 bits.
 * edges: G (lo, hi) pairs. Returns 0, or -1 on bad arguments. */
int kvqo_quantize(const uint16_t* x, int64_t x_row_stride, uint8_t* codes, uint16_t* scales,
                  int64_t L, int H, int D, const int32_t* edges, int G, int bits, int threads) {
  if (L < 0 || H <= 0 || D <= 0 || D > 1024 || (D & 1) || G <= 0 || (bits != 4 && bits != 8))
    return -1;
  if (threads < 1) threads = 1;
  if (threads > KVQO_MAX_THREADS) threads = KVQO_MAX_THREADS;
  if (threads > L) threads = (int)(L > 0 ? L : 1);
  qjob_t jobs[KVQO_MAX_THREADS];
  pthread_t tid[KVQO_MAX_THREADS];
  for (int i = 0; i < threads; ++i) {
    qjob_t j = {x, x_row_stride, codes, scales, L * i / threads, L * (i + 1) / threads,
                H, D, G, bits, edges};
    jobs[i] = j;
  }
  for (int i = 1; i < threads; ++i) pthread_create(&tid[i], NULL, q_thread, &jobs[i]);
  quantize_rows(&jobs[0]);
  for (int i = 1; i < threads; ++i) pthread_join(tid[i], NULL);
  return 0;
}

int kvqo_dequantize(const uint8_t* codes, const uint16_t* scales, uint16_t* out, int64_t L,
                    int H, int D, const int32_t* edges, int G, int bits, int threads) {
  if (L < 0 || H <= 0 || D <= 0 || D > 1024 || (D & 1) || G <= 0 || (bits != 4 && bits != 8))
    return -1;
  if (threads < 1) threads = 1;
  if (threads > KVQO_MAX_THREADS) threads = KVQO_MAX_THREADS;
  if (threads > L) threads = (int)(L > 0 ? L : 1);
  djob_t jobs[KVQO_MAX_THREADS];
  pthread_t tid[KVQO_MAX_THREADS];
  for (int i = 0; i < threads; ++i) {
    djob_t j = {codes, scales, out, L * i / threads, L * (i + 1) / threads, H, D, G, bits, edges};
    jobs[i] = j;
  }
  for (int i = 1; i < threads; ++i) pthread_create(&tid[i], NULL, d_thread, &jobs[i]);
  dequantize_rows(&jobs[0]);
  for (int i = 1; i < threads; ++i) pthread_join(tid[i], NULL);
  return 0;
}

/* ------------------------------------------------------------------------- exhaustive check
 * Reference code of x in a group whose |max| is amax (quant_kv.py:151-153):
 *   s = fl(amax / qmax), s = 1 if amax == 0, code = clamp(rne(fl(x / s)), -qmax, qmax).
 * Kernel formula (no division per element):
 *   s = fl(amax / qmax) (one IEEE divide per group), r = RN(1 / s) (one correctly
 *   rounded reciprocal per group), then per element the Markstein refinement
 *   y0 = RN(x * r), rem = RN(x - y0 * s) (exact, one FMA), y1 = RN(y0 + rem * r)
 *   (one FMA) and code = rne(y1); the exact divide only for groups whose amax is
 *   below `exact_below` (tiny scales, where 1/s overflows or rem underflows).
 *   With exact_below = 2^-100 the count is zero for qmax 7 and 127.
 * Counts the pairs where the two disagree; positive x only (both formulas are odd
 * in x). Returns the number of mismatches and stores the first one in *first. */
typedef struct {
  int qmax;
  uint32_t a0, a1; /* amax bit-pattern range (positive finite bf16) */
  float exact_below;
  int any_rcp;
  long long mismatches;
  uint32_t first;
} xjob_t;

static void* exhaustive_thread(void* p) {
  xjob_t* j = (xjob_t*)p;
  j->mismatches = 0;
  j->first = 0xFFFFFFFFu;
  for (uint32_t ab = j->a0; ab < j->a1; ++ab) {
    float amax = bf16_to_f32((uint16_t)ab);
    float s = amax / (float)j->qmax;
    if (!(s > 0.0f)) s = 1.0f;
    float r = 1.0f / s;
    int fast = amax >= j->exact_below;
    for (uint32_t xb = 0; xb <= ab; ++xb) {
      float x = bf16_to_f32((uint16_t)xb);
      float ref = nearbyintf(x / s);
      if (ref > j->qmax) ref = (float)j->qmax;
      float got;
      if (fast && j->any_rcp) {
        /* the same with each reciprocal within 1 ulp of 1/s: RN(1/s) and both
         * neighbours; a mismatch for any of them counts */
        const float rs[3] = {r, nextafterf(r, 0.0f), nextafterf(r, INFINITY)};
        got = ref;
        for (int k = 0; k < 3; ++k) {
          float y0 = x * rs[k];
          float rem = fmaf(-y0, s, x);
          float g = nearbyintf(fmaf(rem, rs[k], y0));
          if (g > j->qmax) g = (float)j->qmax;
          if (g != ref) got = g;
        }
      } else if (fast) {
        /* Markstein refinement: y0 = RN(x*r), rem = x - y0*s exactly (FMA),
         * y1 = RN(y0 + rem*r) = RN(x/s) when r = RN(1/s). */
        float y0 = x * r;
        float rem = fmaf(-y0, s, x);
        got = nearbyintf(fmaf(rem, r, y0));
      } else {
        got = nearbyintf(x / s);
      }
      if (got > j->qmax) got = (float)j->qmax;
      if (got != ref) {
        if (j->mismatches == 0) j->first = (ab << 16) | xb;
        j->mismatches++;
      }
    }
  }
  return NULL;
}

long long kvqo_check_fast_codes_rcp(int qmax, float exact_below, int any_rcp, int threads, uint32_t* first);
long long kvqo_check_fast_codes(int qmax, float exact_below, int threads, uint32_t* first) {
  return kvqo_check_fast_codes_rcp(qmax, exact_below, 0, threads, first);
}

/* any_rcp != 0: the per-element formula must hold for every reciprocal within
 * one ulp of 1/s (RN(1/s) and its two neighbours), so an approximate reciprocal
 * refined to 1-ulp accuracy may be used. */
long long kvqo_check_fast_codes_rcp(int qmax, float exact_below, int any_rcp, int threads, uint32_t* first) {
  if (threads < 1) threads = 1;
  if (threads > 64) threads = 64;
  xjob_t jobs[64];
  pthread_t tid[64];
  /* positive finite bf16: 0x0000 .. 0x7F7F; split by work (triangular) */
  const uint32_t top = 0x7F80;
  for (int i = 0; i < threads; ++i) {
    double f0 = sqrt((double)i / threads), f1 = sqrt((double)(i + 1) / threads);
    jobs[i].qmax = qmax;
    jobs[i].a0 = (uint32_t)(f0 * top);
    jobs[i].a1 = (i == threads - 1) ? top : (uint32_t)(f1 * top);
    jobs[i].exact_below = exact_below;
    jobs[i].any_rcp = any_rcp;
  }
  for (int i = 0; i < threads; ++i) pthread_create(&tid[i], NULL, exhaustive_thread, &jobs[i]);
  long long total = 0;
  uint32_t f = 0xFFFFFFFFu;
  for (int i = 0; i < threads; ++i) {
    pthread_join(tid[i], NULL);
    total += jobs[i].mismatches;
    if (jobs[i].mismatches && f == 0xFFFFFFFFu) f = jobs[i].first;
  }
  if (first) *first = f;
  return total;
}

/* ------------------------------------------------------------------------- exhaustive check
 * Group scale without a divide: the kernel computes s = amax / qmax as
 *   r = RN(1/qmax), q0 = RN(amax * r), rem = RN(amax - q0 * qmax) (FMA),
 *   s = RN(q0 + rem * r) (FMA)
 * and this returns the number of positive finite bf16 amax for which that
 * differs from the IEEE quotient RN(amax / qmax) (quant_kv.py:151). */
long long kvqo_check_scale_div(int qmax) {
  const float r = 1.0f / (float)qmax;
  long long bad = 0;
  for (uint32_t ab = 1; ab < 0x7F80u; ++ab) {
    float amax = bf16_to_f32((uint16_t)ab);
    float ref = amax / (float)qmax;
    float q0 = amax * r;
    float rem = fmaf(-q0, (float)qmax, amax);
    float s = fmaf(rem, r, q0);
    if (s != ref) bad++;
  }
  return bad;
}
